// K1 on the 5th-generation tensor cores: codebook scoring with the top-a /
// top-b code selection fused into the epilogue.
//
// Reference: ssa/router.py:116-141 -- cosine scores of every routed query /
// key against every code of its KV head's codebook, then topk.  The score
// matrix [rows, N_c] is never written to memory here: each 128-row tile's
// scores live in TMEM one 256-code chunk at a time and are reduced to a
// per-row top-K list by the epilogue warps.
//
// Precision: routed vectors and codes are unit vectors in fp32.  Each is split
// into an f16 pair hi + lo (hi = f16(x), lo = f16(x - hi)); one kind::f16 MMA
// with K = 3*d_s evaluates  a_hi.c_hi + a_lo.c_hi + a_hi.c_lo  with fp32
// accumulation, which carries ~22 significant bits -- close enough to fp32
// that code selection agrees with an fp32/fp64 evaluation except at genuine
// near-ties.  A row = [a_hi | a_lo | a_hi], B row = [c_hi | c_hi | c_lo].
//
// CTA layout (one persistent CTA per SM, static round-robin over tiles):
//   warp 0      producer: 1-D bulk copies (cp.async.bulk) of pre-laid-out
//               codebook chunks into a 3-stage shared-memory ring;
//   warp 1      TMEM allocation and the single-thread tcgen05.mma issuer
//               (M=128, N=256, K=16 per instruction) into a double-buffered
//               accumulator (2 x 256 TMEM columns);
//   warps 2-9   epilogue, two warpgroups: each thread owns one row (TMEM lane)
//               and half of every chunk's columns; tcgen05.ld -> register
//               top-K list; the two halves merge at the end of the tile.
//               The same warps build the next tile's A operand in shared
//               memory while the current tile's MMAs run.
// Operands use the K-major SWIZZLE_NONE canonical layout: 8-row x 16-byte
// core matrices, SBO = 128 B between 8-row groups, LBO between 16-byte K
// groups.
//
// Every wait is bounded (about one second); on expiry the CTA records an
// error bit, stops issuing work, waits (bounded) for its copies and MMAs in
// flight, frees TMEM and exits.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_utils.cuh"

namespace ssa {
namespace tc {

constexpr int kM = 128;
constexpr int kN = 256;
constexpr int kStages = 2;
constexpr int kBufs = 512 / kN;   // TMEM accumulator buffers (all 512 columns)
constexpr int kCand = 32;          // pass-2 candidates buffered per thread (one full batch)
constexpr int kEpiWG = 2;
constexpr int kEpiWarps = 4 * kEpiWG;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kColsPerWG = kN / kEpiWG;
static_assert((kColsPerWG / 32) % 2 == 0, "pass 1 reads two 32-column parts per step");
static_assert(kEpiWG == 2, "the bound merges exactly two lists per row");
template <int DS>
struct Geo {
  static constexpr int K = 3 * DS;
  static constexpr int KG = K / 8;                 // 16-byte K groups per row
  static constexpr int KSTEPS = K / 16;            // MMA instructions per chunk
  static constexpr int A_LBO = (kM / 8) * 128;
  static constexpr int B_LBO = (kN / 8) * 128;
  static constexpr int A_BYTES = kM * K * 2;
  static constexpr int B_BYTES = kN * K * 2;
};

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, N=256, M=128.
constexpr uint32_t kIdesc = idesc_f16(kM, kN, false);
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t ad, uint64_t bd, uint32_t acc) {
  tc::mma_f16(tmem_d, ad, bd, kIdesc, acc);
}

// (hi - l, lo - l) of the fp32 pair (lo, hi) against l = (l, l) packed in 64
// bits: one packed f32x2 subtraction, round to nearest, no flush to zero.
__device__ __forceinline__ uint64_t sub_f32x2(uint32_t lo, uint32_t hi, uint64_t l) {
  const uint64_t a = (static_cast<uint64_t>(hi) << 32) | lo;
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(l));
  return d;
}

// Three-input maximum (one instruction on sm_100; NaN inputs are ignored as by fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// v[j] for a run-time j in [0, 32) without indexing the register array (which
// would move it to local memory): a binary tree of selects on the bits of j.
__device__ __forceinline__ uint32_t select32(const uint32_t (&v)[32], int j) {
  uint32_t w[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) w[t] = (j & 1) ? v[2 * t + 1] : v[2 * t];
#pragma unroll
  for (int t = 0; t < 8; ++t) w[t] = (j & 2) ? w[2 * t + 1] : w[2 * t];
#pragma unroll
  for (int t = 0; t < 4; ++t) w[t] = (j & 4) ? w[2 * t + 1] : w[2 * t];
#pragma unroll
  for (int t = 0; t < 2; ++t) w[t] = (j & 8) ? w[2 * t + 1] : w[2 * t];
  return (j & 16) ? w[1] : w[0];
}

// a[0..N) in descending order: bitonic network, fully unrolled (N a power of two).
template <int N>
__device__ __forceinline__ void sort_desc(float (&a)[N]) {
#pragma unroll
  for (int k = 2; k <= N; k <<= 1)
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int l = i ^ j;
        if (l > i) {
          const float x = a[i], y = a[l];
          const bool desc = (i & k) == 0;
          a[i] = desc ? fmaxf(x, y) : fminf(x, y);
          a[l] = desc ? fminf(x, y) : fmaxf(x, y);
        }
      }
}

// Insert kv into the descending list key[0..K) (its last entry drops out).
// Every position is computed from the old list, key'[t] = max(key[t],
// min(kv, key[t-1])) with key[-1] = +inf, so the dependency depth is two
// compare-selects rather than a chain through all K positions.
template <int K>
__device__ __forceinline__ void insert_desc(uint64_t (&key)[K], uint64_t kv) {
  uint64_t prev = ~0ull;
#pragma unroll
  for (int t = 0; t < K; ++t) {
    const uint64_t cur = key[t];
    const uint64_t m = kv < prev ? kv : prev;
    key[t] = cur > m ? cur : m;
    prev = cur;
  }
}

// Byte offset of element k of row r in a K-major SWIZZLE_NONE image whose K
// groups are LBO bytes apart.
__device__ __forceinline__ uint32_t img_off(int r, int kgroup, int lbo) {
  return static_cast<uint32_t>(kgroup * lbo + (r >> 3) * 128 + (r & 7) * 16);
}

template <int DS, int KMAX>
__global__ void __launch_bounds__(kThreads, 1) code_score_tc_kernel(CodeScoreTcParams p) {
  using G = Geo<DS>;
  constexpr int HI_KSTEPS = DS / 16;                      // pass 1: a_hi . c_hi only
  constexpr uint32_t HI_BYTES = (DS / 8) * G::B_LBO;      // the c_hi third of a chunk image
  constexpr int EPI = 32 * kEpiWarps;                     // epilogue threads
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* a_img = base;                                        // 2 x A_BYTES
  unsigned char* b_img = a_img + 2 * G::A_BYTES;                      // kStages x B_BYTES
  // [kCand][EPI] pass-2 candidate keys; after the last flush the same bytes
  // hold the merge lists ([kEpiWG-1][KMAX][kM] keys, row-minor: conflict-free).
  uint64_t* cand = reinterpret_cast<uint64_t*>(b_img + kStages * G::B_BYTES);
  uint64_t* merge_k = cand;
  __half* lists = reinterpret_cast<__half*>(cand + kCand * EPI);     // [kEpiWG][KMAX][kM] bound lists
  uint64_t* bars = reinterpret_cast<uint64_t*>(lists + kEpiWG * kM * KMAX);
  // barriers: b_full[kStages], b_empty[kStages], t_full[kBufs], t_empty[kBufs], a_ready[2], m_bar[2]
  const uint32_t b_full = smem_u32(bars);
  const uint32_t b_empty = b_full + 8 * kStages;
  const uint32_t t_full = b_empty + 8 * kStages;
  const uint32_t t_empty = t_full + 8 * kBufs;
  const uint32_t a_ready = t_empty + 8 * kBufs;
  const uint32_t m_bar = a_ready + 16;           // epilogue-only barriers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 2 * kBufs + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int chunks = p.n_codes / kN;
  const int64_t total_tiles = p.batch_heads * p.tiles_per_head;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    for (int b = 0; b < kBufs; ++b) {
      mbar_init(t_full + 8 * b, 1);
      mbar_init(t_empty + 8 * b, kEpiWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(a_ready + 8 * b, kEpiWarps);
      mbar_init(m_bar + 8 * b, kEpiWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kBufs * kN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto fail = [&]() {
    *abort_flag = 1;
    if (p.error) atomicOr(p.error, 0x100);
  };
  // barrier of the epilogue warps only (mbarrier, bounded wait)
  auto epi_sync = [&](uint32_t bar, uint32_t parity) {
    __syncwarp();
    if ((threadIdx.x % kWarp) == 0) mbar_arrive(bar);
    return mbar_wait(bar, parity);
  };

  if (warp == 0) {
    // ---------------- producer: every tile streams its codebook twice ----------------
    if (lane == 0) {
      int64_t g = 0;
      bool stop = false;
      for (int64_t tile = blockIdx.x; tile < total_tiles && !stop; tile += gridDim.x) {
        const int64_t bh = tile / p.tiles_per_head;
        const int h = static_cast<int>(bh % p.h_kv);
        const int cbh = p.codebook_heads == 1 ? 0 : h;
        const unsigned char* src = p.image + static_cast<int64_t>(cbh) * chunks * G::B_BYTES;
        for (int pass = 0; pass < 2 && !stop; ++pass) {
          const uint32_t bytes = pass == 0 ? HI_BYTES : static_cast<uint32_t>(G::B_BYTES);
          for (int c = 0; c < chunks; ++c, ++g) {
            const int s = static_cast<int>(g % kStages);
            const uint32_t ph = static_cast<uint32_t>((g / kStages) & 1);
            if (*abort_flag || !mbar_wait(b_empty + 8 * s, ph ^ 1u)) { fail(); stop = true; break; }
            mbar_expect_tx(b_full + 8 * s, bytes);
            bulk_g2s(smem_u32(b_img + s * G::B_BYTES), src + static_cast<int64_t>(c) * G::B_BYTES, bytes,
                     b_full + 8 * s);
          }
        }
      }
      // drain: every issued copy must have landed before the CTA exits
      for (int64_t r = g - 1; r >= 0 && r >= g - kStages; --r) {
        const int s = static_cast<int>(r % kStages);
        mbar_wait(b_full + 8 * s, static_cast<uint32_t>((r / kStages) & 1));
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int64_t g = 0, tl = 0;
      bool issued = false, stop = false;
      for (int64_t tile = blockIdx.x; tile < total_tiles && !stop; tile += gridDim.x, ++tl) {
        const int ab = static_cast<int>(tl & 1);
        if (!mbar_wait(a_ready + 8 * ab, static_cast<uint32_t>((tl >> 1) & 1))) { fail(); break; }
        fence_after();
        const uint32_t a_base = smem_u32(a_img + ab * G::A_BYTES);
        for (int pass = 0; pass < 2 && !stop; ++pass) {
          const int ksteps = pass == 0 ? HI_KSTEPS : G::KSTEPS;
          for (int c = 0; c < chunks; ++c, ++g) {
            const int s = static_cast<int>(g % kStages);
            const int buf = static_cast<int>(g % kBufs);
            if (*abort_flag || !mbar_wait(b_full + 8 * s, static_cast<uint32_t>((g / kStages) & 1)) ||
                !mbar_wait(t_empty + 8 * buf, static_cast<uint32_t>(((g / kBufs) & 1) ^ 1))) {
              fail();
              stop = true;
              break;
            }
            fence_after();
            const uint32_t b_base = smem_u32(b_img + s * G::B_BYTES);
            const uint32_t d = tmem_base + static_cast<uint32_t>(buf * kN);
            for (int ks = 0; ks < ksteps; ++ks) {
              const uint64_t ad = sdesc(a_base + ks * 2 * G::A_LBO, G::A_LBO, 128);
              const uint64_t bd = sdesc(b_base + ks * 2 * G::B_LBO, G::B_LBO, 128);
              mma_f16(d, ad, bd, ks > 0 ? 1u : 0u);
            }
            mma_commit(b_empty + 8 * s);
            mma_commit(t_full + 8 * buf);
            issued = true;
          }
        }
      }
      if (issued) {   // the last commit covers every MMA issued: wait before TMEM is freed
        const int64_t r = g - 1;
        mbar_wait(t_full + 8 * (r % kBufs), static_cast<uint32_t>((r / kBufs) & 1));
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int et = threadIdx.x - 64;              // epilogue thread 0..EPI-1
    const int ew = warp - 2;
    const int wg = ew / 4;
    const int quarter = warp & 3;                 // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;            // row within the tile
    const float inv_t = 1.0f / p.temperature;
    const bool unit_t = p.temperature == 1.0f;

    auto build_a = [&](int64_t tile, int ab) {
      const int64_t bh = tile / p.tiles_per_head;
      const int64_t i = (tile % p.tiles_per_head) * kM + r;
      const bool valid = i < p.n_rows;
      float x[DS];
      if (valid) {
        const float4* src = reinterpret_cast<const float4*>(p.route + (bh * p.n_rows + i) * DS);
#pragma unroll
        for (int e = 0; e < DS / 4; ++e) {
          const float4 t = src[e];
          x[4 * e] = t.x; x[4 * e + 1] = t.y; x[4 * e + 2] = t.z; x[4 * e + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < DS; ++e) x[e] = 0.f;
      }
      unsigned char* img = a_img + ab * G::A_BYTES;
      // K groups: [0, DS/8) hi, [DS/8, 2DS/8) lo, [2DS/8, 3DS/8) hi
#pragma unroll
      for (int kg = 0; kg < G::KG; ++kg) {
        if (kg % kEpiWG != wg) continue;
        const int part = kg / (DS / 8);
        const int e0 = (kg % (DS / 8)) * 8;
        uint32_t w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          __half h2[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float v = x[e0 + 2 * t + u];
            const __half hi = __float2half_rn(v);
            h2[u] = part == 1 ? __float2half_rn(v - __half2float(hi)) : hi;
          }
          w[t] = static_cast<uint32_t>(__half_as_ushort(h2[0])) |
                 (static_cast<uint32_t>(__half_as_ushort(h2[1])) << 16);
        }
        *reinterpret_cast<uint4*>(img + img_off(r, kg, G::A_LBO)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(a_ready + 8 * ab);
    };

    // wait for accumulator chunk g and return its TMEM address for this thread
    auto acquire = [&](int64_t gg, uint32_t& taddr) -> bool {
      const int buf = static_cast<int>(gg % kBufs);
      if (*abort_flag || !mbar_wait(t_full + 8 * buf, static_cast<uint32_t>((gg / kBufs) & 1))) return false;
      fence_after();
      taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
              static_cast<uint32_t>(buf * kN + wg * kColsPerWG);
      return true;
    };
    auto release = [&](int64_t gg) {
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(t_empty + 8 * (gg % kBufs));
    };

    int64_t g = 0, tl = 0;
    int msync = 0;                                 // epilogue barrier uses (parity source)
    if (static_cast<int64_t>(blockIdx.x) < total_tiles) build_a(blockIdx.x, 0);
    for (int64_t tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tl) {
      if (*abort_flag) break;
      const int64_t next = tile + gridDim.x;
      if (next < total_tiles) build_a(next, static_cast<int>((tl + 1) & 1));
      bool ok = true;

      // ---- pass 1: maximum of each of 32 column groups on the a_hi . c_hi scores ----
      float m1[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) m1[j] = -INFINITY;
      for (int c = 0; c < chunks && ok; ++c, ++g) {
        uint32_t taddr;
        if (!acquire(g, taddr)) { ok = false; break; }
#pragma unroll 1
        for (int part = 0; part < kColsPerWG / 32; part += 2) {
          uint32_t v[32], w[32];
          tmem_ld32_async(taddr + part * 32, v);
          tmem_ld32_async(taddr + part * 32 + 32, w);
          tmem_wait();
          if (part == kColsPerWG / 32 - 2) release(g);
#pragma unroll
          for (int j = 0; j < 32; ++j) m1[j] = fmax3(m1[j], __uint_as_float(v[j]), __uint_as_float(w[j]));
        }
      }
      if (!ok) { fail(); break; }
      // The row's 64 column groups (32 per warpgroup, disjoint) have maxima
      // m_1 >= m_2 >= ...: KMAX distinct scores reach m_KMAX, so (up to the
      // dropped lo terms) m_KMAX is a lower bound on the row's KMAX-th largest
      // score.  Each thread sorts its own 32 maxima down to a top-KMAX list,
      // the two lists of a row meet in shared memory (rounded down to f16,
      // which only lowers the bound), and both threads take the KMAX-th
      // largest of their union.
      {
        __half* mine = lists + wg * KMAX * kM + r;     // element t at mine[t * kM]
        // in registers: 15 stages of independent compare-exchanges (an
        // insertion of the 32 maxima into a KMAX-list would chain 32 * KMAX)
        sort_desc(m1);
#pragma unroll
        for (int t = 0; t < KMAX; ++t) mine[t * kM] = __float2half_rd(m1[t]);
      }
      if (!epi_sync(m_bar + 8 * (msync & 1), static_cast<uint32_t>((msync >> 1) & 1))) { fail(); break; }
      ++msync;
      // KMAX-th largest of the union of two descending lists a, b:
      // max over t of min(a[t-1], b[KMAX-1-t]), a[-1] = b[-1] = +inf.  Both
      // warpgroups evaluate it in the same order, so they get the same value.
      float lb;
      {
        const __half* la = lists + r;
        const __half* lo = lists + KMAX * kM + r;
        lb = fmaxf(__half2float(la[(KMAX - 1) * kM]), __half2float(lo[(KMAX - 1) * kM]));
#pragma unroll
        for (int t = 1; t < KMAX; ++t)
          lb = fmaxf(lb, fminf(__half2float(la[(t - 1) * kM]), __half2float(lo[(KMAX - 1 - t) * kM])));
      }
      // |a.c - a_hi.c_hi| <= 2^-10 for unit vectors a, c (f16 rounding of each
      // operand, Cauchy-Schwarz); 2^-9 leaves a margin for fp32 accumulation.
      lb -= 1.0f / 512.0f;
      // strictly below lb (and below +0 when lb is +0), so that the sign of
      // v - lb_below is clear exactly when v >= lb_below
      const float lb_below = lb - fabsf(lb) * 0x1p-20f - 0x1p-126f;
      const uint64_t lb_pair = (static_cast<uint64_t>(__float_as_uint(lb_below)) << 32) | __float_as_uint(lb_below);

      // ---- pass 2: full-precision scores; keep those >= lb (a superset) ----
      TopList<KMAX> top;
      top.init();
      int ncand = 0;
      auto flush = [&]() {
#pragma unroll 1
        for (int t = 0; t < ncand; ++t) {
          const uint64_t kv = cand[t * EPI + et];
          if (kv > top.key[KMAX - 1]) insert_desc(top.key, kv);
        }
        ncand = 0;
      };
      for (int c = 0; c < chunks && ok; ++c, ++g) {
        uint32_t taddr;
        if (!acquire(g, taddr)) { ok = false; break; }
        const int col_base = c * kN + wg * kColsPerWG;
#pragma unroll 1
        for (int part = 0; part < kColsPerWG / 32; ++part) {
          uint32_t v[32];
          tmem_ld32_async(taddr + part * 32, v);
          tmem_wait();
          if (part == kColsPerWG / 32 - 1) release(g);
          // hit bit j <=> v[j] - lb_below >= 0: the sign bits of the 32
          // differences, shifted into one word (two instructions a column).
          // Four independent 8-bit chains, joined at the end, keep the
          // dependency depth at 8 shifts instead of 32.  lb_below < lb, so
          // the hits include every score >= lb; a NaN score may set its bit
          // and is dropped below.
          // The subtractions run two columns per instruction (packed f32x2,
          // round to nearest as the scalar form).
          uint32_t mb[4] = {0u, 0u, 0u, 0u};
#pragma unroll
          for (int j = 3; j >= 0; --j)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint64_t d = sub_f32x2(v[8 * q + 2 * j], v[8 * q + 2 * j + 1], lb_pair);
              mb[q] = __funnelshift_l(static_cast<uint32_t>(d >> 32), mb[q], 1);
              mb[q] = __funnelshift_l(static_cast<uint32_t>(d), mb[q], 1);
            }
          const uint32_t miss = mb[0] | (mb[1] << 8) | (mb[2] << 16) | (mb[3] << 24);
          uint32_t hit = ~miss;
          if (hit) {
            if (ncand + __popc(hit) > kCand) flush();      // the only flush site: keeps code small
            // Hits are rare (about KMAX per row over all of its columns), so
            // each one is taken by a bit scan and a 5-level select on its
            // column rather than by a test of all 32 columns.
#pragma unroll 1
            while (hit) {
              const int j = __ffs(hit) - 1;
              hit &= hit - 1;
              const float x = __uint_as_float(select32(v, j));
              if (x == x) {
                cand[ncand * EPI + et] =
                    rank_key(unit_t ? x : x * inv_t, static_cast<uint32_t>(col_base + part * 32 + j));
                ++ncand;
              }
            }
          }
        }
      }
      if (!ok) { fail(); break; }
      flush();
      // every thread's candidates are consumed before the buffer holds merge lists
      if (!epi_sync(m_bar + 8 * (msync & 1), static_cast<uint32_t>((msync >> 1) & 1))) { fail(); break; }
      ++msync;
      // merge the warpgroups' lists (ranking keys are unique: plain key inserts)
      if (wg > 0) {
#pragma unroll
        for (int t = 0; t < KMAX; ++t) merge_k[((wg - 1) * KMAX + t) * kM + r] = top.key[t];
      }
      if (!epi_sync(m_bar + 8 * (msync & 1), static_cast<uint32_t>((msync >> 1) & 1))) { fail(); break; }
      ++msync;
      if (wg == 0) {
        // top-KMAX of two descending lists of distinct keys: the larger of
        // a[t] and b[KMAX-1-t] forms a bitonic sequence holding exactly the
        // KMAX largest; log2(KMAX) half-cleaner stages sort it
        const uint64_t* other = merge_k + r;
#pragma unroll
        for (int t = 0; t < KMAX; ++t) {
          const uint64_t b = other[(KMAX - 1 - t) * kM];
          top.key[t] = top.key[t] > b ? top.key[t] : b;
        }
#pragma unroll
        for (int j = KMAX / 2; j > 0; j >>= 1)
#pragma unroll
          for (int t = 0; t < KMAX; ++t) {
            const int l = t ^ j;
            if (l > t) {
              const uint64_t x = top.key[t], y = top.key[l];
              top.key[t] = x > y ? x : y;
              top.key[l] = x > y ? y : x;
            }
          }
        const int64_t bh = tile / p.tiles_per_head;
        const int64_t i = (tile % p.tiles_per_head) * kM + r;
        if (i < p.n_rows) {
          const int h = static_cast<int>(bh % p.h_kv);
          const int64_t bat = bh / p.h_kv;
          int32_t* out = p.codes + ((bat * p.n_rows + i) * p.h_kv + h) * p.kk;
#pragma unroll
          for (int t = 0; t < KMAX; ++t)
            if (t < p.kk) out[t] = top.index(t);
        }
      }
      // the bound lists and merge buffers are rewritten next tile only after every
      // epilogue warp is past this point
      if (!epi_sync(m_bar + 8 * (msync & 1), static_cast<uint32_t>((msync >> 1) & 1))) { fail(); break; }
      ++msync;
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kBufs * kN));
  }
}

// Codebook chunk images: for head h and chunk c, the B operand of one MMA
// chunk in the K-major SWIZZLE_NONE layout, rows = codes, K = [hi | hi | lo].
template <int DS>
__global__ void codebook_image_kernel(const float* cbn, unsigned char* img, int64_t heads, int n_codes) {
  using G = Geo<DS>;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= heads * n_codes) return;
  const int64_t h = t / n_codes;
  const int code = static_cast<int>(t % n_codes);
  const int chunk = code / kN, rr = code % kN;
  const float* x = cbn + t * DS;
  unsigned char* dst = img + (h * (n_codes / kN) + chunk) * static_cast<int64_t>(G::B_BYTES);
  for (int kg = 0; kg < G::KG; ++kg) {
    const int part = kg / (DS / 8);
    const int e0 = (kg % (DS / 8)) * 8;
    uint32_t w[4];
    for (int q = 0; q < 4; ++q) {
      __half h2[2];
      for (int u = 0; u < 2; ++u) {
        const float v = x[e0 + 2 * q + u];
        const __half hi = __float2half_rn(v);
        h2[u] = part == 2 ? __float2half_rn(v - __half2float(hi)) : hi;
      }
      w[q] = static_cast<uint32_t>(__half_as_ushort(h2[0])) |
             (static_cast<uint32_t>(__half_as_ushort(h2[1])) << 16);
    }
    *reinterpret_cast<uint4*>(dst + img_off(rr, kg, G::B_LBO)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int DS>
size_t smem_bytes(int kmax) {
  using G = Geo<DS>;
  const size_t shared = std::max<size_t>(static_cast<size_t>(kCand) * 32 * kEpiWarps * 8,
                                         static_cast<size_t>(kEpiWG - 1) * kM * kmax * 8);
  return 1024 + 2 * G::A_BYTES + kStages * G::B_BYTES + shared + static_cast<size_t>(kEpiWG) * kM * kmax * 2 +
         (2 * kStages + 2 * kBufs + 4) * 8 + 16;
}

}  // namespace tc

bool code_score_tc_supported(int d_s, int n_codes) {
  return (d_s == 16 || d_s == 32) && n_codes % tc::kN == 0 && n_codes >= tc::kN;
}

size_t codebook_image_bytes(int heads, int n_codes, int d_s) {
  return static_cast<size_t>(heads) * n_codes * 3 * d_s * 2;
}

cudaError_t launch_codebook_image(const float* cbn, void* img, int heads, int n_codes, int d_s,
                                  cudaStream_t st) {
  const int64_t n = static_cast<int64_t>(heads) * n_codes;
  const unsigned blocks = static_cast<unsigned>(cdiv(n, 256));
  if (d_s == 16) tc::codebook_image_kernel<16><<<blocks, 256, 0, st>>>(cbn, static_cast<unsigned char*>(img), heads, n_codes);
  else tc::codebook_image_kernel<32><<<blocks, 256, 0, st>>>(cbn, static_cast<unsigned char*>(img), heads, n_codes);
  return cudaGetLastError();
}

template <int DS, int KMAX>
static cudaError_t launch_tc(const CodeScoreTcParams& p, cudaStream_t st) {
  const size_t smem = tc::smem_bytes<DS>(KMAX);
  auto kern = tc::code_score_tc_kernel<DS, KMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = p.batch_heads * p.tiles_per_head;
  const unsigned grid = static_cast<unsigned>(tiles < sms ? tiles : sms);
  if (grid == 0) return cudaSuccess;
  kern<<<grid, tc::kThreads, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_code_score_tc(const CodeScoreTcParams& p, int d_s, cudaStream_t st) {
  if (d_s == 32) {
    if (p.kk <= 4) return launch_tc<32, 4>(p, st);
    if (p.kk <= 8) return launch_tc<32, 8>(p, st);
    if (p.kk <= 16) return launch_tc<32, 16>(p, st);
    return launch_tc<32, 32>(p, st);
  }
  if (p.kk <= 4) return launch_tc<16, 4>(p, st);
  if (p.kk <= 8) return launch_tc<16, 8>(p, st);
  if (p.kk <= 16) return launch_tc<16, 16>(p, st);
  return launch_tc<16, 32>(p, st);
}

}  // namespace ssa
