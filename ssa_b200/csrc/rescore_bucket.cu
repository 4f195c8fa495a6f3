// K3, bucket-major path for 16-bit inputs (d 64 or 128, b = 4, packed index).
//
// Same contract as the walking kernel (rescore_mma.cu; ssa/router.py:151-259:
// candidates = keys sharing a code with the query, j <= i when causal, each
// counted once; ranked by qbar . k_j with the lower key index first among
// equal scores; canonical filler; zero padding), and the same result bit for
// bit: the scores come from the same tensor-core fragments in the same order,
// and the selection, sort and output are the shared code of rescore_unit.cuh.
//
// What changes is the order of the work.  The walking kernel gathers every
// candidate key row once per query that reaches it: a key sits in b buckets
// and is a candidate of about a*b*n / (2 N_c) later queries, so each key row
// crosses L2 -> SM a few hundred times.  Here the queries holding code c and
// the keys holding code c meet in one tile: a bucket's key rows are staged in
// shared memory once, its queries stream past them 8 at a time, and each
// score goes to the query's candidate segment in HBM.  Stages:
//   1. qbar_kernel: each unit's group-mean query, split into 16-bit hi and lo
//      rows (the A operand the walking kernel builds in registers);
//   2. the code -> query-row index of the query codes (index.cu's builder);
//   3. locate_kernel: per unit, the causal length of each of its a buckets and
//      their offsets in the unit's segment; segments are claimed from a
//      cursor, and a unit whose segment does not fit the buffer is left to the
//      walking kernel;
//   4. bucket_score_kernel: per (sequence, head, code) bucket, scores on
//      mma.sync m16n8k16 (A rows 0-7 the hi rows of 8 queries, rows 8-15 their
//      lo rows; B the staged key rows), the causal and first-match filters,
//      and the ranking key (or 0 for a dropped entry) into each segment;
//   5. select_kernel: per unit, its segment compacted into shared memory (or
//      read in place when it holds more than CAP keys), then select, sort and
//      write (rescore_unit.cuh).
#include "rescore_unit.cuh"

namespace ssa {

namespace {

constexpr int kKeysPerChunk = 64;    // key rows staged per bucket pass
constexpr int kScoreWarps = 4;       // warps of a bucket CTA (8 queries each at a time)
constexpr int kLocateWarps = 8;      // warps of a locate CTA ...
constexpr int kLocateUnits = 4;      // ... and the units each handles: one claim per 32 units
constexpr int kSelectWarps = 4;

__device__ __forceinline__ int64_t unit_of(const RescoreParams& p, int bh, int i) {
  return static_cast<int64_t>(bh) * p.n_q + i;
}

// --- 1. group-mean query rows -----------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(8 * kWarp) qbar_kernel(RescoreParams p, int64_t units) {
  __shared__ float qs_all[8][D];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t u = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (u >= units) return;
  const int bh = static_cast<int>(u / p.n_q), i = static_cast<int>(u % p.n_q);
  const int bat = bh / p.h_kv, h = bh % p.h_kv;
  float* qs = qs_all[warp];
  group_mean_smem<T, D>(p, bat, i, h, lane, qs);
  uint32_t* hi = reinterpret_cast<uint32_t*>(static_cast<T*>(p.qbar) + u * 2 * D);
  uint32_t* lo = hi + D / 2;
#pragma unroll
  for (int m = lane; m < D / 2; m += kWarp) {
    uint32_t h2, l2;
    split2<T>(qs[2 * m], qs[2 * m + 1], h2, l2);
    hi[m] = h2;
    lo[m] = l2;
  }
}

// --- 3. bucket lengths and segments -------------------------------------------
// Lane t < a of a unit's lanes: the t-th code of the unit, the causal length of
// its key bucket (0 for a code outside [0, n_codes) -- which also sets
// SSA_DEVICE_BAD_CODE -- and for a repeat of an earlier code, whose keys the
// first-match rule drops anyway), part[t] = the lengths before it, part[a] =
// the total.  With a <= 16 (HALF) each half-warp takes a unit, so that two
// units' index searches are in flight together.
template <bool HALF>
__global__ void __launch_bounds__(kLocateWarps * kWarp) locate_kernel(RescoreParams p, int64_t units) {
  constexpr int UPW = HALF ? 2 : 1;                              // units a warp takes at a time
  constexpr int W = kWarp / UPW;                                 // lanes of a unit
  constexpr int SLOTS = kLocateWarps * kLocateUnits * UPW;       // units of the CTA: one claim
  static_assert(SLOTS <= 2 * kWarp, "the claim scans two words a lane");
  __shared__ int totals[SLOTS];
  __shared__ long long bases[SLOTS];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int sub = lane / W, sl = lane % W;
  const bool bad_index = p.index_bad && *p.index_bad != 0;
  const int a = p.a;
  for (int r = 0; r < kLocateUnits; ++r) {
    const int slot = (warp * kLocateUnits + r) * UPW + sub;
    const int64_t u = static_cast<int64_t>(blockIdx.x) * SLOTS + slot;
    const bool live = u < units && !bad_index;
    const int bh = live ? static_cast<int>(u / p.n_q) : 0, i = live ? static_cast<int>(u % p.n_q) : 0;
    const int bat = bh / p.h_kv, h = bh % p.h_kv;
    int len = 0, raw = -1;
    if (live && sl < a) raw = p.q_codes[((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * a + sl];
    // lanes of the same unit holding the same code value
    const unsigned long long tag = (static_cast<unsigned long long>(sub) << 32) | static_cast<unsigned>(raw);
    const unsigned same = __match_any_sync(0xffffffffu, tag);
    if (live && sl < a) {
      const bool valid = static_cast<unsigned>(raw) < static_cast<unsigned>(p.n_codes);
      if (!valid) set_status(p.status, SSA_DEVICE_BAD_CODE);
      const bool first = (same & ((1u << lane) - 1u)) == 0;     // lower lanes of the unit: slots < t
      if (valid && first) {
        int lo, hi;
        bucket_range(p, bh, raw, lo, hi);
        if (p.causal) hi = first_above(bucket_base(p, bh), lo, hi, seg_pos(p.seg, i));
        len = hi - lo;
      }
    }
    int incl = len;
#pragma unroll
    for (int o = 1; o < W; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o, W);
      if (sl >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, a - 1, W);
    if (live) {
      int32_t* part = p.part + u * (a + 1);
      if (sl < a) part[sl] = incl - len;
      if (sl == 0) part[a] = total;
    }
    if (sl == 0) totals[slot] = live ? total : 0;
  }
  __syncthreads();
  // one claim for the CTA's units; offsets in unit order within it
  if (warp == 0) {
    const int v0 = lane < SLOTS ? totals[lane] : 0;
    const int v1 = kWarp + lane < SLOTS ? totals[kWarp + lane] : 0;
    long long i0 = v0, i1 = v1;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const long long y0 = __shfl_up_sync(0xffffffffu, i0, o);
      const long long y1 = __shfl_up_sync(0xffffffffu, i1, o);
      if (lane >= o) {
        i0 += y0;
        i1 += y1;
      }
    }
    const long long t0 = __shfl_sync(0xffffffffu, i0, kWarp - 1);
    unsigned long long base = 0;
    if (lane == kWarp - 1) base = atomicAdd(p.cursor, static_cast<unsigned long long>(i0 + i1));
    base = __shfl_sync(0xffffffffu, base, kWarp - 1);
    if (lane < SLOTS) bases[lane] = static_cast<long long>(base) + (i0 - v0);
    if (kWarp + lane < SLOTS) bases[kWarp + lane] = static_cast<long long>(base) + t0 + (i1 - v1);
  }
  __syncthreads();
  if (threadIdx.x < SLOTS) {
    const int slot = threadIdx.x;
    const int64_t u = static_cast<int64_t>(blockIdx.x) * SLOTS + slot;
    if (u < units) {
      const long long off = bases[slot];
      p.seg_off[u] = (!bad_index && off + totals[slot] <= p.cand_capacity) ? off : -1;
    }
  }
}

// --- 4. bucket tiles ----------------------------------------------------------
// The first-match rule drops a key reached through code c at slot t of a query
// when one of the query's codes before slot t is also a code of the key.  Per
// chunk of staged keys, an open-addressed table maps every code the keys hold
// besides c to the bit set of the keys holding it; a query row ORs the sets of
// its codes before t and drops exactly the keys in the union.
constexpr int kTableSlots = 512;                     // >= 2.6x the 3 * 64 codes a chunk inserts
static_assert(kTableSlots >= 2 * 3 * kKeysPerChunk, "code table load factor");

template <int D>
struct BucketSmem {
  uint4 krow[kKeysPerChunk * D / 8];             // key rows, 16-byte chunks XOR-swizzled by row
  int32_t kidx[kKeysPerChunk];                   // key positions
  int32_t tcode[kTableSlots];                    // code table: code (-1 = empty) ...
  uint32_t tkeys[kTableSlots][kKeysPerChunk / 32];  // ... and the chunk's keys that hold it
};

__device__ __forceinline__ unsigned code_slot(int code) {
  return (static_cast<unsigned>(code) * 0x9E3779B1u) >> (32 - 9);
}

template <typename T, int D>
__global__ void __launch_bounds__(kScoreWarps * kWarp) bucket_score_kernel(RescoreParams p) {
  constexpr int CH = D / 8;            // 16-byte chunks per row
  constexpr int KP = D / 32;           // pairs of k-steps
  constexpr int KW = kKeysPerChunk / 32;
  static_assert(kTableSlots == 512, "code_slot takes 9 bits");
  static_assert(KW == 2, "the drop set is two words");
  extern __shared__ __align__(128) unsigned char dyn[];
  BucketSmem<D>& s = *reinterpret_cast<BucketSmem<D>*>(dyn);
  if (p.index_bad && *p.index_bad != 0) return;
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int gid = lane >> 2, tig = lane & 3;
  const int bh = static_cast<int>(blockIdx.x / p.n_codes), c = static_cast<int>(blockIdx.x % p.n_codes);
  const int bat = bh / p.h_kv, h = bh % p.h_kv;
  const int a = p.a;
  int klo, khi;
  bucket_range(p, bh, c, klo, khi);
  const int32_t* qptr = p.q_ptr + static_cast<int64_t>(bh) * (p.n_codes + 1);
  const int qlo = qptr[c], nq = qptr[c + 1] - qlo;
  const int nk = khi - klo;
  if (nq <= 0 || nk <= 0) return;
  const int32_t* qents = p.q_rows + static_cast<int64_t>(bh) * p.n_q * a + qlo;
  const int32_t* bkeys = bucket_base(p, bh) + klo;
  const int4* bcodes = p.bucket_codes + static_cast<int64_t>(bh) * p.entry_stride + klo;
  const T* kbase = static_cast<const T*>(p.k) + bat * p.k_sb + static_cast<int64_t>(h) * p.k_sh;
  const T* qbar = static_cast<const T*>(p.qbar);

  for (int k0 = 0; k0 < nk; k0 += kKeysPerChunk) {
    const int kn = min(kKeysPerChunk, nk - k0);
    __syncthreads();                                        // the previous chunk is no longer read
    for (int slot = threadIdx.x; slot < kTableSlots; slot += blockDim.x) {
      s.tcode[slot] = -1;
#pragma unroll
      for (int w = 0; w < KW; ++w) s.tkeys[slot][w] = 0u;
    }
    for (int r = threadIdx.x; r < kn; r += blockDim.x) s.kidx[r] = bkeys[k0 + r];
    __syncthreads();
    // the table: each key's codes other than c (a code outside the codebook
    // is inserted like any other value; it matches no valid query code)
    for (int r = threadIdx.x; r < kn; r += blockDim.x) {
      const int4 c4 = bcodes[k0 + r];
      const int codes[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int x = codes[q];
        if (x == c) continue;
        unsigned slot = code_slot(x);
        while (true) {                                      // fewer than half the slots are taken
          const int prev = atomicCAS(&s.tcode[slot], -1, x);
          if (prev == -1 || prev == x) break;
          slot = (slot + 1) & (kTableSlots - 1);
        }
        atomicOr(&s.tkeys[slot][r >> 5], 1u << (r & 31));
      }
    }
    for (int idx = threadIdx.x; idx < kn * CH; idx += blockDim.x) {
      const int r = idx / CH, ch = idx % CH;
      s.krow[r * CH + (ch ^ (r & 7))] =
          __ldg(reinterpret_cast<const uint4*>(kbase + static_cast<int64_t>(s.kidx[r]) * p.k_sn + ch * 8));
    }
    __syncthreads();

    // the query index holds entry numbers e = row * a + t: query row e / a
    // has code c in its slot t = e % a.  A warp takes 8 entries (rows) at a
    // time, lane (gid, tig) working on entry gid; the next group's entry
    // numbers are loaded while the current group is scored.
    int next_e = warp * 8 + gid < nq ? qents[warp * 8 + gid] : -1;
    for (int g0 = warp * 8; g0 < nq; g0 += kScoreWarps * 8) {
      const int e = next_e;
      next_e = g0 + kScoreWarps * 8 + gid < nq ? qents[g0 + kScoreWarps * 8 + gid] : -1;
      const bool in_group = e >= 0;
      const int qi = in_group ? e / a : 0, row_t = in_group ? e % a : 0;
      const int64_t row_u = unit_of(p, bh, qi);
      // the row's A fragments, its segment and the part of it that belongs
      // to this bucket
      uint4 hi4[KP], lo4[KP];
      {
        const T* qr = qbar + row_u * 2 * D + 8 * tig;
#pragma unroll
        for (int kp = 0; kp < KP; ++kp) {
          hi4[kp] = in_group ? __ldg(reinterpret_cast<const uint4*>(qr + kp * 32)) : make_uint4(0, 0, 0, 0);
          lo4[kp] = in_group ? __ldg(reinterpret_cast<const uint4*>(qr + D + kp * 32)) : make_uint4(0, 0, 0, 0);
        }
      }
      // the row's codes before slot t (a quarter of them a lane), loaded in
      // the same round trip as its segment and part
      int early[8];
      {
        const int32_t* qcodes = p.q_codes + ((static_cast<int64_t>(bat) * p.n_q + qi) * p.h_kv + h) * a;
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const int t = tig + 4 * m;
          early[m] = in_group && t < row_t ? qcodes[t] : -1;
        }
      }
      int row_m = 0;
      int64_t row_dst = 0;
      if (in_group) {
        const int64_t off = p.seg_off[row_u];
        const int32_t* part = p.part + row_u * (a + 1);
        const int ps = part[row_t];
        const int pe = part[row_t + 1];
        if (off >= 0) {
          row_m = pe - ps;
          row_dst = off + ps;
        }
      }
      // the keys of this chunk the row reaches through an earlier code: the
      // quad looks up the row's codes before slot t, a quarter each
      uint32_t drop[KW];
#pragma unroll
      for (int w = 0; w < KW; ++w) drop[w] = 0u;
      if (row_m > k0 && row_t > 0) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          if (tig + 4 * m >= row_t) break;
          const int x = early[m];
          unsigned slot = code_slot(x);
          while (true) {                                    // ends at x or at an empty slot
            const int tc = s.tcode[slot];
            if (tc == x) {
#pragma unroll
              for (int w = 0; w < KW; ++w) drop[w] |= s.tkeys[slot][w];
              break;
            }
            if (tc == -1) break;
            slot = (slot + 1) & (kTableSlots - 1);
          }
        }
      }
#pragma unroll
      for (int w = 0; w < KW; ++w) {
        drop[w] |= __shfl_xor_sync(0xffffffffu, drop[w], 1);
        drop[w] |= __shfl_xor_sync(0xffffffffu, drop[w], 2);
      }
      int mmax = row_m;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mmax = max(mmax, __shfl_xor_sync(0xffffffffu, mmax, o));
      if (mmax <= k0) continue;                             // every row's keys end before this chunk
      const bool live = row_m > k0;
      uint32_t qa[2 * KP][4];
#pragma unroll
      for (int kp = 0; kp < KP; ++kp) {
        if (!live) hi4[kp] = lo4[kp] = make_uint4(0, 0, 0, 0);
        qa[2 * kp][0] = hi4[kp].x; qa[2 * kp][1] = lo4[kp].x; qa[2 * kp][2] = hi4[kp].y; qa[2 * kp][3] = lo4[kp].y;
        qa[2 * kp + 1][0] = hi4[kp].z; qa[2 * kp + 1][1] = lo4[kp].z;
        qa[2 * kp + 1][2] = hi4[kp].w; qa[2 * kp + 1][3] = lo4[kp].w;
      }
      const int kend = min(kn, mmax - k0);                  // keys of this chunk some row needs
      uint64_t* dst = p.cand + row_dst;
      for (int nt = 0; nt * 8 < kend; ++nt) {
        const int kr = nt * 8 + gid;                        // B: key row kr of the chunk
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kp = 0; kp < KP; ++kp) {
          const uint4 v = s.krow[kr * CH + ((4 * kp + tig) ^ (kr & 7))];
          mma16816<T>(sc, qa[2 * kp], v.x, v.y);
          mma16816<T>(sc, qa[2 * kp + 1], v.z, v.w);
        }
        if (live) {
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int col = nt * 8 + 2 * tig + e2;          // key of the chunk for output column e2
            const int colg = k0 + col;
            if (col < kn && colg < row_m) {
              const uint32_t dw = col < 32 ? drop[0] : drop[1];
              const bool keep = ((dw >> (col & 31)) & 1u) == 0u;
              dst[colg] = keep ? rank_key(sc[e2] + sc[2 + e2], static_cast<uint32_t>(s.kidx[col])) : 0ull;
            }
          }
        }
      }
    }
  }
}

// --- 5. per-unit selection -------------------------------------------------------
// CAP keys of a unit are compacted into shared memory; SEL >= k is the room
// for the selected ones.
template <int CAP, int SEL>
__global__ void __launch_bounds__(kSelectWarps * kWarp) select_kernel(RescoreParams p, int64_t units) {
  using Smem = RsMmaSmem<CAP, SEL>;
  extern __shared__ __align__(128) unsigned char dyn[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  Smem& s = reinterpret_cast<Smem*>(dyn)[warp];
  // warps take the units head by head, largest positions (most candidates)
  // first, so that the launch does not end on a tail of heavy units
  const int64_t w = static_cast<int64_t>(blockIdx.x) * kSelectWarps + warp;
  if (w >= units) return;
  const int bh = static_cast<int>(w / p.n_q), i = p.n_q - 1 - static_cast<int>(w % p.n_q);
  const int64_t u = unit_of(p, bh, i);
  const int bat = bh / p.h_kv, h = bh % p.h_kv;
  if (rescore_skip_bad_index(p, bat, i, h, lane, kWarp)) return;
  const int64_t off = p.seg_off[u];
  if (off < 0) {
    // no room in the buffer: the walking kernel's second tier takes the unit
    // (its numbering: head-major, positions descending)
    if (lane == 0) p.ovf2_list[atomicAdd(p.ovf2_count, 1)] = static_cast<int32_t>(bh * p.n_q + (p.n_q - 1 - i));
    return;
  }
  const int total = p.part[u * (p.a + 1) + p.a];
  const uint64_t* seg = p.cand + off;
  const int k_eff = min(p.top_k, p.n);
  const int64_t row = (static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h;
  constexpr int kAhead = 4;                                  // segment loads in flight per lane
  int count = 0;
  if (total > CAP) {
    for (int idx0 = 0; idx0 < total; idx0 += kAhead * kWarp) {
      uint64_t kv[kAhead];
#pragma unroll
      for (int r = 0; r < kAhead; ++r) {
        const int idx = idx0 + r * kWarp + lane;
        kv[r] = idx < total ? seg[idx] : 0ull;
      }
#pragma unroll
      for (int r = 0; r < kAhead; ++r) count += __popc(__ballot_sync(0xffffffffu, kv[r] != 0ull));
    }
    if (count > CAP) {                                       // select straight from the segment
      select_sort_write(p, s, seg, total, count, k_eff, lane, row);
      return;
    }
    count = 0;
  }
  for (int idx0 = 0; idx0 < total; idx0 += kAhead * kWarp) {
    uint64_t kv[kAhead];
#pragma unroll
    for (int r = 0; r < kAhead; ++r) {
      const int idx = idx0 + r * kWarp + lane;
      kv[r] = idx < total ? seg[idx] : 0ull;
    }
#pragma unroll
    for (int r = 0; r < kAhead; ++r) {
      const unsigned bal = __ballot_sync(0xffffffffu, kv[r] != 0ull);
      if (kv[r] != 0ull) s.keys[count + __popc(bal & ((1u << lane) - 1u))] = kv[r];
      count += __popc(bal);
    }
  }
  __syncwarp();
  select_sort_write(p, s, s.keys, count, count, k_eff, lane, row);
}

template <int CAP, int SEL>
cudaError_t launch_select(const RescoreParams& p, int64_t units, cudaStream_t st) {
  const size_t smem = sizeof(RsMmaSmem<CAP, SEL>) * kSelectWarps;
  auto kern = select_kernel<CAP, SEL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  kern<<<static_cast<unsigned>(cdiv(units, kSelectWarps)), kSelectWarps * kWarp, smem, st>>>(p, units);
  return cudaGetLastError();
}

}  // namespace

bool rescore_bucket_supported(int d, int a, int b, int k_eff, bool packed_index, ssa_dtype dt) {
  return (dt == SSA_BF16 || dt == SSA_F16) && (d == 64 || d == 128) && b == 4 && a >= 1 && a <= 32 &&
         k_eff <= kMaxSel && packed_index;
}

template <typename T, int D>
cudaError_t launch_rescore_bucket(const RescoreParams& p, cudaStream_t st) {
  const int64_t units = static_cast<int64_t>(p.batch) * p.h_kv * p.n_q;
  if (units == 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(p.cursor, 0, sizeof(unsigned long long), st);
  if (e != cudaSuccess) return e;
  qbar_kernel<T, D><<<static_cast<unsigned>(cdiv(units, 8)), 8 * kWarp, 0, st>>>(p, units);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  IndexParams ip{};
  ip.k_codes = p.q_codes;
  ip.bucket_ptr = p.q_ptr;
  ip.bucket_keys = p.q_rows;
  ip.counts = p.q_counts;
  ip.partials = p.q_partials;
  ip.status = p.status;
  ip.k_codes_sb = static_cast<int64_t>(p.n_q) * p.h_kv * p.a;
  ip.batch = p.batch;
  ip.n = p.n_q;
  ip.h_kv = p.h_kv;
  ip.b = p.a;
  ip.n_codes = p.n_codes;
  ip.tile_keys = index_tile_keys(p.a);
  ip.tiles = static_cast<int>(cdiv(p.n_q, ip.tile_keys));
  ip.chunks = cdiv(static_cast<int64_t>(p.n_codes) * ip.tiles, kScanChunk);
  ip.store_entry = 1;
  e = launch_build_index(ip, st);
  if (e != cudaSuccess) return e;
  constexpr int per_cta = kLocateWarps * kLocateUnits;
  if (p.a <= kWarp / 2)
    locate_kernel<true><<<static_cast<unsigned>(cdiv(units, 2 * per_cta)), kLocateWarps * kWarp, 0, st>>>(p, units);
  else
    locate_kernel<false><<<static_cast<unsigned>(cdiv(units, per_cta)), kLocateWarps * kWarp, 0, st>>>(p, units);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const size_t smem = sizeof(BucketSmem<D>);
  e = cudaFuncSetAttribute(bucket_score_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const int64_t buckets = static_cast<int64_t>(p.batch) * p.h_kv * p.n_codes;
  bucket_score_kernel<T, D><<<static_cast<unsigned>(buckets), kScoreWarps * kWarp, smem, st>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int k_eff = std::min(p.top_k, p.n);
  if (k_eff > 256) return launch_select<1024, kMaxSel>(p, units, st);
  if (k_eff > 128) return launch_select<512, 256>(p, units, st);
  return launch_select<512, 128>(p, units, st);
}

template cudaError_t launch_rescore_bucket<__nv_bfloat16, 64>(const RescoreParams&, cudaStream_t);
template cudaError_t launch_rescore_bucket<__nv_bfloat16, 128>(const RescoreParams&, cudaStream_t);
template cudaError_t launch_rescore_bucket<__half, 64>(const RescoreParams&, cudaStream_t);
template cudaError_t launch_rescore_bucket<__half, 128>(const RescoreParams&, cudaStream_t);

}  // namespace ssa
