// K3: per (query i, KV head h) candidate union, causal filter, full-dimension
// re-score, top-k, canonical filler and zero padding.
//
// Reference: CodebookRouter._select_candidates, ssa/router.py:151-214, and
// _build_candidate_mask, ssa/router.py:216-259.  The reference scores every
// key (an [n, h_kv, g, n] tensor), masks non-candidates and future keys with
// -inf and runs topk over all n.  Only the candidates matter, so this kernel
// walks the query's a code buckets of the inverted index instead:
//
//   candidates(i,h) = U_t bucket(q_codes[i,h,t])  (restricted to j <= i if causal)
//   score(j)        = qbar_i . k_j,   qbar_i = mean_g q[i, h*g+g']
//
// qbar . k_j equals the reference's group mean of per-head logits
// (ssa/router.py:191) up to rounding; the common 1/sqrt(d) factor does not
// change the order.  Ranking key: (score desc, key index asc) -- the
// reference's topk with a fixed tie rule.  Fewer than min(k, n) candidates are
// followed by the lowest-index non-candidate keys in index order (the -inf
// entries of the reference's topk, ssa/router.py:200-204), then zero padding
// when k > n (ssa/router.py:206-211).
//
// A key reached through several of the query's codes is kept only from the
// first such code in the query's code order (first-match rule), which needs
// only the key's own b codes -- no per-query hash set.
//
// One CTA of 128 threads per (bat, i, h).  Candidates' 64-bit ranking keys
// collect in shared memory (capacity `cap`, a power of two >= min(k, n)); a
// bitonic sort orders them.  If a query has more than `cap` distinct
// candidates, a radix select over re-enumerated candidates finds the k-th key
// first and only the top k are collected.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace ssa {

constexpr int kRsThreads = 128;
constexpr int kMaxCodesPerQuery = 32;

struct RsStatic {
  int32_t qc[kMaxCodesPerQuery];
  int32_t lo[kMaxCodesPerQuery];
  int32_t pre[kMaxCodesPerQuery + 1];
  uint32_t count;
  uint32_t hist[256];
  uint32_t warp_sums[kRsThreads / kWarp];
  uint64_t prefix;
  uint32_t remaining;
  int done;
};

size_t rescore_smem_bytes(int cap, int top_k) {
  // keys[cap] (u64) + qbar[d<=256] (f32) + bitmap + per-word zero prefix
  const size_t words = static_cast<size_t>(cdiv(top_k, 32));
  return static_cast<size_t>(cap) * 8 + 256 * 4 + words * 4 * 2;
}

template <typename T>
struct RsUnit {
  const RescoreParams& p;
  RsStatic& s;
  const float* qbar;
  const int32_t* bk;       // bucket keys of (bat, h)
  const int32_t* kcodes;   // k_codes of bat
  const T* kbase;          // k of (bat, h)
  int h;
  int a;

  __device__ __forceinline__ float score(int32_t j) const {
    const T* row = kbase + static_cast<int64_t>(j) * p.k_sn;
    float acc0 = 0.f, acc1 = 0.f;
    for (int e = 0; e < p.d; e += 8) {
      float f[8];
      load8<T>(row + e, f);
      const float4 q0 = *reinterpret_cast<const float4*>(qbar + e);
      const float4 q1 = *reinterpret_cast<const float4*>(qbar + e + 4);
      acc0 = fmaf(f[0], q0.x, acc0); acc1 = fmaf(f[1], q0.y, acc1);
      acc0 = fmaf(f[2], q0.z, acc0); acc1 = fmaf(f[3], q0.w, acc1);
      acc0 = fmaf(f[4], q1.x, acc0); acc1 = fmaf(f[5], q1.y, acc1);
      acc0 = fmaf(f[6], q1.z, acc0); acc1 = fmaf(f[7], q1.w, acc1);
    }
    return acc0 + acc1;
  }

  // Calls f(key) for every distinct candidate of this unit.
  template <class F>
  __device__ __forceinline__ void enumerate(F f) const {
    const int total = s.pre[a];
    int t = 0;
    for (int m = threadIdx.x; m < total; m += kRsThreads) {
      while (s.pre[t + 1] <= m) ++t;
      const int32_t j = bk[s.lo[t] + (m - s.pre[t])];
      // first-match dedupe: skip if one of the query's earlier codes is also one of j's codes
      bool dup = false;
      if (t > 0) {
        const int32_t* jc = kcodes + (static_cast<int64_t>(j) * p.h_kv + h) * p.b;
        for (int x = 0; x < p.b && !dup; ++x) {
          const int32_t c = jc[x];
          for (int u = 0; u < t; ++u) dup |= (s.qc[u] == c);
        }
      }
      if (dup) continue;
      f(rank_key(score(j), static_cast<uint32_t>(j)));
    }
  }
};

__device__ __forceinline__ void bitonic_sort_desc(uint64_t* keys, int size) {
  for (int k2 = 2; k2 <= size; k2 <<= 1) {
    for (int j = k2 >> 1; j > 0; j >>= 1) {
      for (int e = threadIdx.x; e < size; e += blockDim.x) {
        const int ixj = e ^ j;
        if (ixj > e) {
          const uint64_t x = keys[e], y = keys[ixj];
          const bool desc = (e & k2) == 0;
          if ((x < y) == desc) { keys[e] = y; keys[ixj] = x; }
        }
      }
      __syncthreads();
    }
  }
}

// Unit index -> (bat, h, i): head-major (the K rows of the heads in flight stay
// in L2); within a head the largest query positions first, since causal work
// grows with i.
__device__ __forceinline__ void unit_coords(const RescoreParams& p, int64_t unit, int& bh, int& i) {
  bh = static_cast<int>(unit / p.n_q);
  i = p.n_q - 1 - static_cast<int>(unit % p.n_q);
}

// One unit on a whole CTA (any candidate count, any k): the general path.
template <typename T>
__device__ void rescore_unit_block(const RescoreParams& p, int64_t unit, RsStatic& s, unsigned char* dyn) {
  uint64_t* keys = reinterpret_cast<uint64_t*>(dyn);
  float* qbar = reinterpret_cast<float*>(dyn + static_cast<size_t>(p.cap) * 8);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(qbar + 256);
  uint32_t* zpre = bitmap + cdiv(p.top_k, 32);

  int bh, i;
  unit_coords(p, unit, bh, i);
  const int bat = bh / p.h_kv, h = bh % p.h_kv;
  if (rescore_skip_bad_index(p, bat, i, h, threadIdx.x, blockDim.x)) return;
  const int pos = seg_pos(p.seg, i);
  const int a = p.a;
  const int k_eff = min(p.top_k, p.n);
  const int32_t* bk = bucket_base(p, bh);

  if (threadIdx.x < kWarp) {
    int len = 0;
    if (threadIdx.x < a) {
      const int c = checked_code(p.q_codes[((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * a + threadIdx.x],
                                 p.n_codes, p.status);
      int lo, hi;
      bucket_range(p, bh, c, lo, hi);
      if (p.causal) {  // bucket keys ascend: keep the prefix with j <= pos
        int l = lo, u = hi;
        while (l < u) {
          const int mid = (l + u) >> 1;
          if (bk[mid] <= pos) l = mid + 1; else u = mid;
        }
        hi = l;
      }
      s.qc[threadIdx.x] = c;
      s.lo[threadIdx.x] = lo;
      len = hi - lo;
    }
    int x = len;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (static_cast<int>(threadIdx.x) >= o) x += y;
    }
    if (threadIdx.x < a) s.pre[threadIdx.x + 1] = x;
    if (threadIdx.x == 0) { s.pre[0] = 0; s.count = 0; }
  }
  {
    const T* qrow = static_cast<const T*>(p.q) + bat * p.q_sb + static_cast<int64_t>(i) * p.q_sn +
                    static_cast<int64_t>(h) * p.group * p.q_sh;
    const float inv_g = 1.0f / static_cast<float>(p.group);
    for (int e = threadIdx.x; e < p.d; e += kRsThreads) {
      float acc = 0.f;
      for (int gg = 0; gg < p.group; ++gg) acc += Elem<T>::to_f(qrow[gg * p.q_sh + e]);
      qbar[e] = p.group == 1 ? acc : acc * inv_g;
    }
  }
  __syncthreads();

  RsUnit<T> u{p, s, qbar, bk,
              p.k_codes + static_cast<int64_t>(bat) * p.k_codes_sb,
              static_cast<const T*>(p.k) + bat * p.k_sb + static_cast<int64_t>(h) * p.k_sh, h, a};
  const uint32_t cap = static_cast<uint32_t>(p.cap);
  u.enumerate([&](uint64_t key) {
    const uint32_t slot = atomicAdd(&s.count, 1u);
    if (slot < cap) keys[slot] = key;
  });
  __syncthreads();
  const uint32_t cu = s.count;
  int nsel;
  if (cu <= cap) {
    int size = 1;
    while (size < static_cast<int>(cu)) size <<= 1;
    for (int e = cu + threadIdx.x; e < size; e += kRsThreads) keys[e] = 0ull;
    __syncthreads();
    bitonic_sort_desc(keys, size);
    nsel = min(static_cast<int>(cu), k_eff);
  } else {
    // radix select of the k_eff-th largest key over re-enumerated candidates
    if (threadIdx.x == 0) { s.prefix = 0ull; s.remaining = k_eff; s.done = 0; }
    uint64_t mask = 0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int e = threadIdx.x; e < 256; e += kRsThreads) s.hist[e] = 0;
      __syncthreads();
      const uint64_t prefix = s.prefix;
      u.enumerate([&](uint64_t key) {
        if ((key & mask) == prefix) atomicAdd(&s.hist[(key >> shift) & 255u], 1u);
      });
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t acc = 0;
        int sel = 0;
        for (int dg = 255; dg >= 0; --dg) {
          if (acc + s.hist[dg] >= s.remaining) { sel = dg; break; }
          acc += s.hist[dg];
        }
        s.remaining -= acc;
        s.prefix |= static_cast<uint64_t>(sel) << shift;
        s.done = s.hist[sel] == s.remaining;
      }
      mask |= 255ull << shift;
      __syncthreads();
      if (s.done) break;
    }
    const uint64_t thr = s.prefix;
    __syncthreads();
    if (threadIdx.x == 0) s.count = 0;
    __syncthreads();
    u.enumerate([&](uint64_t key) {
      if (key >= thr) {
        const uint32_t slot = atomicAdd(&s.count, 1u);
        if (slot < cap) keys[slot] = key;
      }
    });
    __syncthreads();
    int size = 1;
    while (size < k_eff) size <<= 1;
    for (int e = k_eff + threadIdx.x; e < size; e += kRsThreads) keys[e] = 0ull;
    __syncthreads();
    bitonic_sort_desc(keys, size);
    nsel = k_eff;
  }

  const int64_t obase = ((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * p.top_k;
  auto put = [&](int slot, int32_t j) {
    if (p.index_i64) static_cast<int64_t*>(p.out)[obase + slot] = j;
    else static_cast<int32_t*>(p.out)[obase + slot] = j;
  };
  for (int e = threadIdx.x; e < nsel; e += kRsThreads) put(e, static_cast<int32_t>(rank_key_index(keys[e])));

  if (static_cast<int>(cu) < k_eff) {
    // filler: the lowest-index keys that are not candidates
    const int need = k_eff - static_cast<int>(cu);
    const int words = static_cast<int>(cdiv(k_eff, 32));
    for (int w = threadIdx.x; w < words; w += kRsThreads) bitmap[w] = 0u;
    __syncthreads();
    for (int e = threadIdx.x; e < static_cast<int>(cu); e += kRsThreads) {
      const uint32_t j = rank_key_index(keys[e]);
      if (j < static_cast<uint32_t>(k_eff)) atomicOr(&bitmap[j >> 5], 1u << (j & 31));
    }
    __syncthreads();
    // exclusive prefix of free (zero) bits per word; thread-serial over words
    // per thread chunk, then a block scan of the chunk sums
    const int per = static_cast<int>(cdiv(words, kRsThreads));
    const int w0 = threadIdx.x * per;
    uint32_t local = 0;
    for (int w = w0; w < min(words, w0 + per); ++w) {
      uint32_t free_bits = ~bitmap[w];
      if (w == words - 1 && (k_eff & 31)) free_bits &= (1u << (k_eff & 31)) - 1u;
      zpre[w] = local;
      local += __popc(free_bits);
    }
    // block exclusive scan of `local`
    const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
    uint32_t x = local;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == kWarp - 1) s.warp_sums[warp] = x;
    __syncthreads();
    uint32_t before = 0;
    for (int w = 0; w < warp; ++w) before += s.warp_sums[w];
    const uint32_t base = before + x - local;
    for (int w = w0; w < min(words, w0 + per); ++w) {
      uint32_t free_bits = ~bitmap[w];
      if (w == words - 1 && (k_eff & 31)) free_bits &= (1u << (k_eff & 31)) - 1u;
      uint32_t rank = base + zpre[w];
      while (free_bits && rank < static_cast<uint32_t>(need)) {
        const int bit = __ffs(free_bits) - 1;
        free_bits &= free_bits - 1;
        put(static_cast<int>(cu) + static_cast<int>(rank), w * 32 + bit);
        ++rank;
      }
    }
  }
  for (int e = k_eff + threadIdx.x; e < p.top_k; e += kRsThreads) put(e, 0);
  if (p.cand_counts && threadIdx.x == 0)
    p.cand_counts[(static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h] = static_cast<int32_t>(cu);
  __syncthreads();   // shared state is reused by the CTA's next unit
}

// General path: every unit (list == nullptr, one CTA each) or the units
// listed by the warp kernels (count read on the device; a persistent grid
// whose CTAs claim the next unclaimed unit through a counter, since the
// listed units differ in cost by several times).
template <typename T>
__global__ void __launch_bounds__(kRsThreads) rescore_block_kernel(RescoreParams p, const int32_t* list,
                                                                  const int32_t* list_count, int32_t* list_next) {
  __shared__ RsStatic s;
  __shared__ int claimed;
  extern __shared__ __align__(16) unsigned char dyn[];
  if (!list) {
    const int64_t n = static_cast<int64_t>(p.batch) * p.n_q * p.h_kv;
    for (int64_t it = blockIdx.x; it < n; it += gridDim.x) rescore_unit_block<T>(p, it, s, dyn);
    return;
  }
  const int n = *list_count;
  while (true) {
    if (threadIdx.x == 0) claimed = atomicAdd(list_next, 1);
    __syncthreads();
    const int it = claimed;
    __syncthreads();                               // read before thread 0 claims again
    if (it >= n) break;
    rescore_unit_block<T>(p, static_cast<int64_t>(list[it]), s, dyn);
  }
}

// ---------------------------------------------------------------------------
// Fast path: one warp per unit, no CTA barriers.  Candidates' ranking keys are
// appended with warp-aggregated slots (ballot + popc) to a per-warp buffer of
// kWarpCap keys and sorted in registers by a warp bitonic network (E keys per
// lane, blocked layout: intra-lane stages are register compare-exchanges,
// inter-lane stages use shuffles).  Units with more than kWarpCap distinct
// candidates, or k > kWarpCap, are appended to an overflow list for the
// general path.
// ---------------------------------------------------------------------------
constexpr int kWarpUnits = 4;
constexpr int kWarpCap = 512;

struct RsWarpSmem {
  __align__(16) float qbar[256];     // read as float4: must stay 16-byte aligned
  uint64_t keys[kWarpCap];
  int32_t qc[kMaxCodesPerQuery];
  int32_t lo[kMaxCodesPerQuery];
  int32_t pre[kMaxCodesPerQuery + 1];
  uint32_t bitmap[kWarpCap / 32];
};

// Descending bitonic sort of 32*E keys in a warp; key[e] of lane l sits at
// position e*32 + l (cyclic layout: loads from and stores to consecutive
// positions are conflict-free / coalesced).  Partners closer than 32
// positions are exchanged with shuffles, farther ones inside the lane.
template <int E>
__device__ __forceinline__ void warp_sort_desc(uint64_t (&key)[E], int lane) {
  constexpr int N = 32 * E;
#pragma unroll
  for (int k2 = 2; k2 <= N; k2 <<= 1) {
#pragma unroll
    for (int j = k2 >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const int f = e ^ (j >> 5);
          if (f > e) {
            const bool desc = ((e * 32 + lane) & k2) == 0;
            const uint64_t x = key[e], y = key[f];
            const bool swap = desc ? (x < y) : (x > y);
            key[e] = swap ? y : x;
            key[f] = swap ? x : y;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint64_t other = __shfl_xor_sync(0xffffffffu, key[e], j);
          const bool desc = ((e * 32 + lane) & k2) == 0;
          const bool lower = (lane & j) == 0;
          const bool keep_max = desc == lower;
          const uint64_t mx = key[e] > other ? key[e] : other;
          const uint64_t mn = key[e] > other ? other : key[e];
          key[e] = keep_max ? mx : mn;
        }
      }
    }
  }
}

template <int E>
__device__ __forceinline__ void warp_sort_emit(const RsWarpSmem& s, int count, int nsel, int lane,
                                               const RescoreParams& p, int64_t obase) {
  uint64_t key[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int idx = e * 32 + lane;
    key[e] = idx < count ? s.keys[idx] : 0ull;
  }
  warp_sort_desc<E>(key, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int idx = e * 32 + lane;
    if (idx < nsel) {
      const int32_t j = static_cast<int32_t>(rank_key_index(key[e]));
      if (p.index_i64) static_cast<int64_t*>(p.out)[obase + idx] = j;
      else static_cast<int32_t*>(p.out)[obase + idx] = j;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarpUnits * kWarp) rescore_warp_kernel(RescoreParams p) {
  __shared__ RsWarpSmem smem[kWarpUnits];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  RsWarpSmem& s = smem[warp];
  const int64_t units = static_cast<int64_t>(p.batch) * p.n_q * p.h_kv;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kWarpUnits + warp;
  if (unit >= units) return;
  int bh, i;
  unit_coords(p, unit, bh, i);
  const int bat = bh / p.h_kv, h = bh % p.h_kv;
  if (rescore_skip_bad_index(p, bat, i, h, lane, kWarp)) return;
  const int pos = seg_pos(p.seg, i);
  const int a = p.a;
  const int k_eff = min(p.top_k, p.n);
  const int32_t* bk = bucket_base(p, bh);

  int len = 0;
  if (lane < a) {
    const int c = checked_code(p.q_codes[((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * a + lane],
                               p.n_codes, p.status);
    int lo, hi;
    bucket_range(p, bh, c, lo, hi);
    if (p.causal) {
      int l = lo, u = hi;
      while (l < u) {
        const int mid = (l + u) >> 1;
        if (bk[mid] <= pos) l = mid + 1; else u = mid;
      }
      hi = l;
    }
    s.qc[lane] = c;
    s.lo[lane] = lo;
    len = hi - lo;
  }
  int x = len;
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane < a) s.pre[lane + 1] = x;
  if (lane == 0) s.pre[0] = 0;
  const int total = __shfl_sync(0xffffffffu, x, a - 1);
  {
    const T* qrow = static_cast<const T*>(p.q) + bat * p.q_sb + static_cast<int64_t>(i) * p.q_sn +
                    static_cast<int64_t>(h) * p.group * p.q_sh;
    const float inv_g = 1.0f / static_cast<float>(p.group);
    for (int e = lane; e < p.d; e += kWarp) {
      float acc = 0.f;
      for (int gg = 0; gg < p.group; ++gg) acc += Elem<T>::to_f(qrow[gg * p.q_sh + e]);
      s.qbar[e] = p.group == 1 ? acc : acc * inv_g;
    }
  }
  __syncwarp();

  const int32_t* kcodes = p.k_codes + static_cast<int64_t>(bat) * p.k_codes_sb;
  const T* kbase = static_cast<const T*>(p.k) + bat * p.k_sb + static_cast<int64_t>(h) * p.k_sh;
  // Two candidates per lane per iteration.  For each, the K row and the key's
  // codes are loaded as soon as the key index is known, so the dedupe test
  // and the dot product share one round trip to L2.
  auto locate = [&](int m, int& t) -> int32_t {
    while (s.pre[t + 1] <= m) ++t;
    return bk[s.lo[t] + (m - s.pre[t])];
  };
  auto is_dup = [&](int32_t j, int t) -> bool {
    bool dup = false;
    if (t > 0) {
      const int32_t* jc = kcodes + (static_cast<int64_t>(j) * p.h_kv + h) * p.b;
      for (int y = 0; y < p.b; ++y) {
        const int32_t c = jc[y];
        for (int u = 0; u < t; ++u) dup |= (s.qc[u] == c);
      }
    }
    return dup;
  };
  int count = 0;
  int t = 0;
  for (int m0 = 0; m0 < total; m0 += 2 * kWarp) {
    const int ma = m0 + lane, mb = ma + kWarp;
    const bool ha = ma < total, hb = mb < total;
    int ta = t;
    const int32_t ja = ha ? locate(ma, ta) : 0;
    int tb = ta;
    const int32_t jb = hb ? locate(mb, tb) : ja;
    t = hb ? tb : ta;
    const T* ra = kbase + static_cast<int64_t>(ja) * p.k_sn;
    const T* rb = kbase + static_cast<int64_t>(jb) * p.k_sn;
    float a0 = 0.f, a1 = 0.f, b0 = 0.f, b1 = 0.f;
    for (int e = 0; e < p.d; e += 8) {
      float fa[8], fb[8];
      load8<T>(ra + e, fa);
      load8<T>(rb + e, fb);
      const float4 q0 = *reinterpret_cast<const float4*>(s.qbar + e);
      const float4 q1 = *reinterpret_cast<const float4*>(s.qbar + e + 4);
      a0 = fmaf(fa[0], q0.x, a0); a1 = fmaf(fa[1], q0.y, a1);
      a0 = fmaf(fa[2], q0.z, a0); a1 = fmaf(fa[3], q0.w, a1);
      a0 = fmaf(fa[4], q1.x, a0); a1 = fmaf(fa[5], q1.y, a1);
      a0 = fmaf(fa[6], q1.z, a0); a1 = fmaf(fa[7], q1.w, a1);
      b0 = fmaf(fb[0], q0.x, b0); b1 = fmaf(fb[1], q0.y, b1);
      b0 = fmaf(fb[2], q0.z, b0); b1 = fmaf(fb[3], q0.w, b1);
      b0 = fmaf(fb[4], q1.x, b0); b1 = fmaf(fb[5], q1.y, b1);
      b0 = fmaf(fb[6], q1.z, b0); b1 = fmaf(fb[7], q1.w, b1);
    }
    const bool keep_a = ha && !is_dup(ja, ta);
    const bool keep_b = hb && !is_dup(jb, tb);
    const unsigned bal_a = __ballot_sync(0xffffffffu, keep_a);
    const unsigned bal_b = __ballot_sync(0xffffffffu, keep_b);
    const unsigned below = (1u << lane) - 1u;
    const int slot_a = count + __popc(bal_a & below);
    const int slot_b = count + __popc(bal_a) + __popc(bal_b & below);
    if (keep_a && slot_a < kWarpCap) s.keys[slot_a] = rank_key(a0 + a1, static_cast<uint32_t>(ja));
    if (keep_b && slot_b < kWarpCap) s.keys[slot_b] = rank_key(b0 + b1, static_cast<uint32_t>(jb));
    count += __popc(bal_a) + __popc(bal_b);
  }
  if (count > kWarpCap || k_eff > kWarpCap) {
    if (lane == 0) p.ovf_list[atomicAdd(p.ovf_count, 1)] = static_cast<int32_t>(unit);
    return;
  }
  __syncwarp();
  const int nsel = min(count, k_eff);
  const int64_t obase = ((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * p.top_k;
  if (count <= 32 * 8) warp_sort_emit<8>(s, count, nsel, lane, p, obase);
  else warp_sort_emit<16>(s, count, nsel, lane, p, obase);
  auto put = [&](int slot, int32_t j) {
    if (p.index_i64) static_cast<int64_t*>(p.out)[obase + slot] = j;
    else static_cast<int32_t*>(p.out)[obase + slot] = j;
  };
  if (count < k_eff) {
    // filler: the lowest-index keys that are not candidates (k_eff <= kWarpCap)
    const int need = k_eff - count;
    const int words = (k_eff + 31) / 32;
    if (lane < words) s.bitmap[lane] = 0u;
    __syncwarp();
    for (int e = lane; e < count; e += kWarp) {
      const uint32_t j = rank_key_index(s.keys[e]);
      if (j < static_cast<uint32_t>(k_eff)) atomicOr(&s.bitmap[j >> 5], 1u << (j & 31));
    }
    __syncwarp();
    uint32_t free_bits = 0;
    if (lane < words) {
      free_bits = ~s.bitmap[lane];
      if (lane == words - 1 && (k_eff & 31)) free_bits &= (1u << (k_eff & 31)) - 1u;
    }
    const int nfree = __popc(free_bits);
    int incl = nfree;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int rank = incl - nfree;
    while (free_bits && rank < need) {
      const int bit = __ffs(free_bits) - 1;
      free_bits &= free_bits - 1;
      put(count + rank, lane * 32 + bit);
      ++rank;
    }
  }
  for (int e = k_eff + lane; e < p.top_k; e += kWarp) put(e, 0);
  if (p.cand_counts && lane == 0)
    p.cand_counts[(static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h] = count;
}

template <typename T>
static cudaError_t launch_rescore_t(const RescoreParams& p, cudaStream_t st) {
  const int64_t units = static_cast<int64_t>(p.batch) * p.n_q * p.h_kv;
  const size_t smem = rescore_smem_bytes(p.cap, p.top_k);
  cudaError_t e = cudaFuncSetAttribute(rescore_block_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  if (std::min(p.top_k, p.n) > kWarpCap || p.ovf_list == nullptr) {
    rescore_block_kernel<T><<<static_cast<unsigned>(units), kRsThreads, smem, st>>>(p, nullptr, nullptr, nullptr);
    return cudaGetLastError();
  }
  e = cudaMemsetAsync(p.ovf_count, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(p.ovf_next, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return e;
  const ssa_dtype dt = sizeof(T) == 4 ? SSA_F32 : (std::is_same<T, __half>::value ? SSA_F16 : SSA_BF16);
  if (rescore_mma_supported(p, dt)) {
    e = launch_rescore_mma(p, dt, st);
    if (e != cudaSuccess) return e;
  } else {
    rescore_warp_kernel<T><<<static_cast<unsigned>(cdiv(units, kWarpUnits)), kWarpUnits * kWarp, 0, st>>>(p);
  }
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rescore_block_kernel<T>, kRsThreads, smem);
  if (e != cudaSuccess) return e;
  const int64_t grid = std::min<int64_t>(units, static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1));
  rescore_block_kernel<T><<<static_cast<unsigned>(grid), kRsThreads, smem, st>>>(p, p.ovf_list, p.ovf_count,
                                                                                  p.ovf_next);
  return cudaGetLastError();
}

cudaError_t launch_rescore(const RescoreParams& p, ssa_dtype dt, cudaStream_t st) {
  const int64_t units = static_cast<int64_t>(p.batch) * p.n_q * p.h_kv;
  if (units == 0) return cudaSuccess;
  if (dt == SSA_F32) return launch_rescore_t<float>(p, st);
  if (dt == SSA_BF16) return launch_rescore_t<__nv_bfloat16>(p, st);
  return launch_rescore_t<__half>(p, st);
}

}  // namespace ssa
