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

constexpr int kKeysPerChunk = 128;   // key rows staged per bucket pass
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
// Lane t < a: the t-th code of the unit, the causal length of its key bucket
// (0 for a code outside [0, n_codes) -- which also sets SSA_DEVICE_BAD_CODE --
// and for a repeat of an earlier code, whose keys the first-match rule drops
// anyway), part[t] = the lengths before it, part[a] = the total.
__global__ void __launch_bounds__(kLocateWarps * kWarp) locate_kernel(RescoreParams p, int64_t units) {
  __shared__ int totals[kLocateWarps * kLocateUnits];
  __shared__ long long bases[kLocateWarps * kLocateUnits];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const bool bad_index = p.index_bad && *p.index_bad != 0;
  const int a = p.a;
  for (int r = 0; r < kLocateUnits; ++r) {
    const int slot = warp * kLocateUnits + r;
    const int64_t u = (static_cast<int64_t>(blockIdx.x) * kLocateWarps + warp) * kLocateUnits + r;
    int total = 0;
    if (u < units && !bad_index) {
      const int bh = static_cast<int>(u / p.n_q), i = static_cast<int>(u % p.n_q);
      const int bat = bh / p.h_kv, h = bh % p.h_kv;
      const int pos = seg_pos(p.seg, i);
      int len = 0, raw = -1;
      if (lane < a) raw = p.q_codes[((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * a + lane];
      const unsigned in_a = a >= kWarp ? 0xffffffffu : ((1u << a) - 1u);
      const unsigned same = __match_any_sync(0xffffffffu, raw) & in_a;
      if (lane < a) {
        const bool valid = static_cast<unsigned>(raw) < static_cast<unsigned>(p.n_codes);
        if (!valid) set_status(p.status, SSA_DEVICE_BAD_CODE);
        const bool first = (same & ((1u << lane) - 1u)) == 0;
        if (valid && first) {
          int lo, hi;
          bucket_range(p, bh, raw, lo, hi);
          if (p.causal) hi = first_above(bucket_base(p, bh), lo, hi, pos);
          len = hi - lo;
        }
      }
      int incl = len;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      int32_t* part = p.part + u * (a + 1);
      if (lane < a) part[lane] = incl - len;
      total = __shfl_sync(0xffffffffu, incl, a - 1);
      if (lane == 0) part[a] = total;
    }
    if (lane == 0) totals[slot] = total;
  }
  __syncthreads();
  // one claim for the CTA's units; offsets in unit order within it
  if (warp == 0) {
    const int v = lane < kLocateWarps * kLocateUnits ? totals[lane] : 0;
    long long incl = v;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    unsigned long long base = 0;
    if (lane == kWarp - 1) base = atomicAdd(p.cursor, static_cast<unsigned long long>(incl));
    base = __shfl_sync(0xffffffffu, base, kWarp - 1);
    if (lane < kLocateWarps * kLocateUnits) bases[lane] = static_cast<long long>(base) + (incl - v);
  }
  __syncthreads();
  if (threadIdx.x < kLocateWarps * kLocateUnits) {
    const int slot = threadIdx.x;
    const int64_t u = (static_cast<int64_t>(blockIdx.x) * kLocateWarps + slot / kLocateUnits) * kLocateUnits +
                      slot % kLocateUnits;
    if (u < units) {
      const long long off = bases[slot];
      p.seg_off[u] = (!bad_index && off + totals[slot] <= p.cand_capacity) ? off : -1;
    }
  }
}

// --- 4. bucket tiles ----------------------------------------------------------
template <int D>
struct BucketSmem {
  uint4 krow[kKeysPerChunk * D / 8];             // key rows, 16-byte chunks XOR-swizzled by row
  int4 kcode[kKeysPerChunk];                     // the b = 4 codes of each key
  uint64_t ksig[kKeysPerChunk];                  // code_bits of each key's other codes
  int32_t kidx[kKeysPerChunk];                   // key positions
  int32_t qc[kScoreWarps][8][33];                // codes of each warp's 8 queries (padded rows)
};

// One bit per code (code mod 64): if the bits of a key's codes other than the
// bucket's and the bits of a query's codes before slot t have nothing in
// common, the two share no code before t and the first-match rule keeps the
// key; otherwise the codes are compared exactly.
__device__ __forceinline__ uint64_t code_bit(int c) { return 1ull << (static_cast<unsigned>(c) & 63u); }

template <typename T, int D>
__global__ void __launch_bounds__(kScoreWarps * kWarp) bucket_score_kernel(RescoreParams p) {
  constexpr int CH = D / 8;            // 16-byte chunks per row
  constexpr int KP = D / 32;           // pairs of k-steps
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
    for (int r = threadIdx.x; r < kn; r += blockDim.x) {
      s.kidx[r] = bkeys[k0 + r];
      const int4 c4 = bcodes[k0 + r];
      s.kcode[r] = c4;
      s.ksig[r] = (c4.x != c ? code_bit(c4.x) : 0ull) | (c4.y != c ? code_bit(c4.y) : 0ull) |
                  (c4.z != c ? code_bit(c4.z) : 0ull) | (c4.w != c ? code_bit(c4.w) : 0ull);
    }
    __syncthreads();
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
      // the row's codes before slot t (first-match rule), its A fragments,
      // its segment and the part of it that belongs to this bucket
      const int32_t* qcodes = p.q_codes + ((static_cast<int64_t>(bat) * p.n_q + qi) * p.h_kv + h) * a;
      uint64_t row_sig = 0ull;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int t = tig + 4 * m;
        if (in_group && t < row_t) {
          const int raw = qcodes[t];
          s.qc[warp][gid][t] = raw;
          row_sig |= code_bit(raw);
        }
      }
      row_sig |= __shfl_xor_sync(0xffffffffu, row_sig, 1);
      row_sig |= __shfl_xor_sync(0xffffffffu, row_sig, 2);
      uint4 hi4[KP], lo4[KP];
      {
        const T* qr = qbar + row_u * 2 * D + 8 * tig;
#pragma unroll
        for (int kp = 0; kp < KP; ++kp) {
          hi4[kp] = in_group ? __ldg(reinterpret_cast<const uint4*>(qr + kp * 32)) : make_uint4(0, 0, 0, 0);
          lo4[kp] = in_group ? __ldg(reinterpret_cast<const uint4*>(qr + D + kp * 32)) : make_uint4(0, 0, 0, 0);
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
      __syncwarp();                                         // s.qc rows are complete
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
      const int32_t* qcr = s.qc[warp][gid];
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
          for (int e = 0; e < 2; ++e) {
            const int col = nt * 8 + 2 * tig + e;            // key of the chunk for output column e
            const int colg = k0 + col;
            if (col < kn && colg < row_m) {
              bool keep = true;
              if (s.ksig[col] & row_sig) {
                const int4 c4 = s.kcode[col];
                for (int uu = 0; uu < row_t; ++uu) {
                  const int32_t q = qcr[uu];
                  keep &= (q != c4.x) & (q != c4.y) & (q != c4.z) & (q != c4.w);
                }
              }
              dst[colg] = keep ? rank_key(sc[e] + sc[2 + e], static_cast<uint32_t>(s.kidx[col])) : 0ull;
            }
          }
        }
      }
      __syncwarp();                                         // qc rows are rewritten by the next group
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
  locate_kernel<<<static_cast<unsigned>(cdiv(units, per_cta)), kLocateWarps * kWarp, 0, st>>>(p, units);
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
