// K3 fast path for 16-bit inputs: one warp per (bat, i, h) unit, candidate
// re-scoring on tensor cores.
//
// Same contract as the CTA-wide path in rescore.cu (ssa/router.py:151-259:
// candidates = keys sharing a code with the query, j <= i when causal;
// ranked by qbar . k_j with the lower key index first among equal scores;
// canonical filler; zero padding).  Steps, all inside one warp:
//   1. the query's a buckets are located (causal cut by an 8-probe search) and
//      walked 128 keys at a time (all loads of a group issued together); the
//      first-match rule drops keys reached through an earlier code; kept key
//      indices are compacted with ballots;
//   2. kept keys are scored 32 at a time on the tensor cores (mma.sync
//      m16n8k16).  B fragments are loaded straight from global memory into
//      registers with 16-byte loads: the reduction (head-dim) axis is
//      permuted identically in A and B so that each lane reads 8 consecutive
//      elements of a key row per pair of k-steps.  The A operand holds qbar
//      split into a 16-bit hi part (row 0) and lo part (row 8); both rows of
//      each output column land in the same thread, so hi + lo gives
//      qbar . k_j with fp32 accuracy;
//   3. if there are more candidates than k, a warp radix select (8 bits per
//      pass over the 64-bit ranking keys, in shared memory) finds the k-th
//      key and the top k are compacted;
//   4. the selected keys are sorted in registers (bitonic, 32*E keys) and
//      written in order; filler and zero padding follow.
// Three tiers: every unit first runs with room for 512 candidates (4 warps per
// CTA); units with more go to an overflow list that a second launch runs with
// room for 1024 (4 warps per CTA, persistent, each warp claiming the next
// unit of the list), and its overflow to a third with room for 2048 (2 warps
// per CTA).  Units beyond that, or with k > 512, go to the CTA-wide path.
// Queries expected to hold far more candidates than the first tier's room
// (long sequences only) start in the second tier.
#include <cmath>

#include "common.cuh"
#include "kernels.cuh"
#include "mma_utils.cuh"

namespace ssa {

#ifndef SSA_RS_UNITS
#define SSA_RS_UNITS 4
#endif
constexpr int kMaxSel = 512;        // k handled on this path
constexpr int kBatch = 32;          // candidates per MMA batch (4 n-tiles)
constexpr int kWalk = 4;            // bucket-walk iterations whose loads are issued together

template <int CAP>
struct __align__(128) RsMmaSmem {
  uint64_t keys[CAP];                          // ranking keys of all candidates
  // kept key indices (CAP int32), then the selected keys (k <= kMaxSel)
  // (its last 1 KB doubles as the radix-select histogram, and before the walk
  // as the group-mean query: neither overlaps a live use of sel)
  uint64_t sel[CAP / 2 > kMaxSel ? CAP / 2 : kMaxSel];
  int32_t qc[32];
  int32_t lo[32];
  int32_t pre[33];
  uint32_t bitmap[kMaxSel / 32];
};

// Descending bitonic sort of 32*E keys, blocked layout: key[e] of lane l is
// at position l*E + e, so the stages with partner distance < E compare within
// a lane and only log2(32) of every log2(32*E) stages shuffle.  The merge
// direction of a stage, (position & k2) == 0, depends only on e while
// k2 < E and only on the lane from k2 = E on, so it is computed once per
// stage (not per element) and every compare-exchange is one 64-bit compare
// and two 64-bit selects.  The stage loops from k2 = 2E on stay rolled
// (run-time distances): the whole network is a few hundred instructions of
// code, so the warps of a CTA do not evict one another's instructions.
template <int E>
__device__ __forceinline__ void cx_desc(uint64_t (&key)[E], int e, int f, bool desc) {
  const uint64_t x = key[e], y = key[f];
  const bool sw = (x > y) != desc;           // equal keys: either order
  key[e] = sw ? y : x;
  key[f] = sw ? x : y;
}

template <int E>
__device__ __forceinline__ void sort_desc_blocked(uint64_t (&key)[E], int lane) {
  constexpr int N = 32 * E;
  // k2 < E: within each lane, direction fixed by e
#pragma unroll
  for (int k2 = 2; k2 < E; k2 <<= 1)
#pragma unroll
    for (int jj = k2 >> 1; jj > 0; jj >>= 1)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if ((e ^ jj) > e) cx_desc<E>(key, e, e ^ jj, (e & k2) == 0);
  // k2 = E: each lane's E keys in the direction of the lane's parity
  {
    const bool desc = (lane & 1) == 0;
#pragma unroll
    for (int jj = E >> 1; jj > 0; jj >>= 1)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if ((e ^ jj) > e) cx_desc<E>(key, e, e ^ jj, desc);
  }
  const int lk = lane * E;
#pragma unroll 1
  for (int k2 = 2 * E; k2 <= N; k2 <<= 1) {
    const bool desc = (lk & k2) == 0;
#pragma unroll 1
    for (int j = k2 >> 1; j >= E; j >>= 1) {       // partner in lane ^ (j / E)
      const bool keep_max = desc == ((lk & j) == 0);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const uint64_t other = __shfl_xor_sync(0xffffffffu, key[e], j / E);
        key[e] = ((key[e] > other) == keep_max) ? key[e] : other;
      }
    }
#pragma unroll
    for (int jj = E >> 1; jj > 0; jj >>= 1)        // partner in the same lane
#pragma unroll
      for (int e = 0; e < E; ++e)
        if ((e ^ jj) > e) cx_desc<E>(key, e, e ^ jj, desc);
  }
}

template <int E>
__device__ __forceinline__ void sort_and_write(const uint64_t* src, int nsel, int lane, const RescoreParams& p,
                                               int64_t obase) {
  uint64_t key[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {              // any input order: read conflict-free
    const int idx = e * 32 + lane;
    key[e] = idx < nsel ? src[idx] : 0ull;
  }
  sort_desc_blocked<E>(key, lane);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int idx = lane * E + e;
    if (idx < nsel) {
      const int32_t j = static_cast<int32_t>(rank_key_index(key[e]));
      if (p.index_i64) static_cast<int64_t*>(p.out)[obase + idx] = j;
      else static_cast<int32_t*>(p.out)[obase + idx] = j;
    }
  }
}

// First index in [l, u) whose key exceeds pos (u if none); keys ascend.  Each
// round trip to memory loads eight probes that cut the range into nine parts,
// so a bucket of a few hundred keys takes two or three round trips instead of
// the eight of a binary search.
__device__ __forceinline__ int first_above(const int32_t* bk, int l, int u, int pos) {
  while (u - l > 8) {
    const int len = u - l;
    int pr[8], v[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) pr[t] = l + ((t + 1) * len) / 9;   // strictly increasing in (l, u)
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = bk[pr[t]];
    // the probes <= pos form a prefix: the answer lies after the last of them
    // and at or before the first probe above pos
    int nl = l, nu = u;
#pragma unroll
    for (int t = 0; t < 8; ++t) nl = v[t] <= pos ? pr[t] + 1 : nl;
#pragma unroll
    for (int t = 7; t >= 0; --t) nu = v[t] > pos ? pr[t] : nu;
    l = nl;
    u = nu;
  }
  int v[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) v[t] = l + t < u ? bk[l + t] : INT_MAX;
  int c = 0;
#pragma unroll
  for (int t = 0; t < 8; ++t) c += v[t] <= pos ? 1 : 0;
  return l + c;
}

template <typename T, int D, int CAP>
__device__ __forceinline__ void rescore_mma_unit(const RescoreParams& p, int64_t unit, RsMmaSmem<CAP>& s,
                                                 int lane, int32_t* out_list, int32_t* out_count) {
  constexpr int KSTEPS = D / 16;
  // head-major, largest query positions first within a head (as the CTA path)
  const int bh = static_cast<int>(unit / p.n_q);
  const int i = p.n_q - 1 - static_cast<int>(unit % p.n_q);
  const int bat = bh / p.h_kv, h = bh % p.h_kv;
  if (rescore_skip_bad_index(p, bat, i, h, lane, kWarp)) return;
  const int pos = seg_pos(p.seg, i);
  const int a = p.a;
  const int k_eff = min(p.top_k, p.n);
  const int32_t* bk = bucket_base(p, bh);
  const int gid = lane >> 2, tig = lane & 3;
  uint32_t* hist = reinterpret_cast<uint32_t*>(s.sel) + (sizeof(s.sel) / 4 - 256);

  // ---- 1a. the query's buckets (causal prefix of each) ----
  int len = 0;
  if (lane < a) {
    const int c = checked_code(p.q_codes[((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * a + lane],
                               p.n_codes, p.status);
    int lo, hi;
    bucket_range(p, bh, c, lo, hi);
    if (p.causal) hi = first_above(bk, lo, hi, pos);
    s.qc[lane] = c;
    s.lo[lane] = lo;
    len = hi - lo;
  }
  int incl = len;
#pragma unroll
  for (int o = 1; o < kWarp; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane < a) s.pre[lane + 1] = incl;
  if (lane == 0) s.pre[0] = 0;
  const int total = __shfl_sync(0xffffffffu, incl, a - 1);

  // ---- qbar as A fragments: row 0 = hi part, row 8 = lo part (lanes 0..3) ----
  // k-step pair kp covers head dims [32kp, 32kp+32); lane tig's 8 dims
  // 32kp+8tig+{0..7} feed (k 2tig..2tig+1, k 2tig+8..2tig+9) of step 2kp and
  // of step 2kp+1, matching the B fragments loaded below.  All lanes load the
  // group's rows together (lane: 8-dim chunk lane % CH of heads lane / CH,
  // + 32 / CH, ...); the chunk sums meet in shared memory.
  uint32_t qa[KSTEPS][4];
  {
    constexpr int CH = D / 8;                     // 8-dim chunks per row
    constexpr int HP = kWarp / CH;                // heads per pass
    constexpr int MAXP = 16 / HP;                 // passes for a group of up to 16 heads
    const T* qrow = static_cast<const T*>(p.q) + bat * p.q_sb + static_cast<int64_t>(i) * p.q_sn +
                    static_cast<int64_t>(h) * p.group * p.q_sh;
    const int ch = lane % CH, h0 = lane / CH;
    float x[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) x[u] = 0.f;
#pragma unroll
    for (int ps = 0; ps < MAXP; ++ps) {
      const int gg = h0 + ps * HP;
      if (gg < p.group) {
        float f[8];
        load8<T>(qrow + static_cast<int64_t>(gg) * p.q_sh + ch * 8, f);
#pragma unroll
        for (int u = 0; u < 8; ++u) x[u] += f[u];
      }
    }
#pragma unroll
    for (int o = CH; o < kWarp; o <<= 1)
#pragma unroll
      for (int u = 0; u < 8; ++u) x[u] += __shfl_xor_sync(0xffffffffu, x[u], o);
    float* qs = reinterpret_cast<float*>(hist);      // D floats; sel is free until the walk
    if (lane < CH) {
      const float inv_g = 1.0f / static_cast<float>(p.group);
#pragma unroll
      for (int u = 0; u < 8; ++u) qs[ch * 8 + u] = p.group != 1 ? x[u] * inv_g : x[u];
    }
    __syncwarp();
#pragma unroll
    for (int kp = 0; kp < KSTEPS / 2; ++kp) {
      qa[2 * kp][0] = qa[2 * kp][1] = qa[2 * kp][2] = qa[2 * kp][3] = 0u;
      qa[2 * kp + 1][0] = qa[2 * kp + 1][1] = qa[2 * kp + 1][2] = qa[2 * kp + 1][3] = 0u;
      if (gid == 0) {
        const float* y = qs + kp * 32 + 8 * tig;
        split2<T>(y[0], y[1], qa[2 * kp][0], qa[2 * kp][1]);
        split2<T>(y[2], y[3], qa[2 * kp][2], qa[2 * kp][3]);
        split2<T>(y[4], y[5], qa[2 * kp + 1][0], qa[2 * kp + 1][1]);
        split2<T>(y[6], y[7], qa[2 * kp + 1][2], qa[2 * kp + 1][3]);
      }
    }
  }
  __syncwarp();

  // ---- 1b. walk the buckets: first-match dedupe, compact kept key indices ----
  const int32_t* kcodes = p.k_codes + static_cast<int64_t>(bat) * p.k_codes_sb;
  int32_t* jlist = reinterpret_cast<int32_t*>(s.sel);
  // with b == 4 the index carries each entry's key codes beside it: key and
  // codes of an entry are loaded in the same round trip
  const int4* bcodes = p.bucket_codes ? p.bucket_codes + static_cast<int64_t>(bh) * p.entry_stride : nullptr;
  int count = 0;
  int t = 0;
  for (int m0 = 0; m0 < total; m0 += kWalk * kWarp) {
    int32_t j[kWalk];
    int tt[kWalk];
    bool keep[kWalk];
    int4 c4[kWalk];
#pragma unroll
    for (int w = 0; w < kWalk; ++w) {          // key indices of the group (coalesced within a bucket)
      const int m = m0 + w * kWarp + lane;
      keep[w] = m < total;
      j[w] = 0;
      c4[w] = make_int4(-1, -1, -1, -1);
      if (keep[w]) {
        while (s.pre[t + 1] <= m) ++t;
        const int e = s.lo[t] + (m - s.pre[t]);
        j[w] = bk[e];
        if (bcodes && t > 0) c4[w] = bcodes[e];
      }
      tt[w] = t;
    }
    if (p.b == 4) {
      if (!bcodes) {
#pragma unroll
        for (int w = 0; w < kWalk; ++w)        // the keys' codes, all loads in flight together
          c4[w] = keep[w] && tt[w] > 0
                      ? *reinterpret_cast<const int4*>(kcodes + (static_cast<int64_t>(j[w]) * p.h_kv + h) * 4)
                      : make_int4(-1, -1, -1, -1);
      }
#pragma unroll
      for (int w = 0; w < kWalk; ++w)
        for (int u = 0; u < tt[w]; ++u) {
          const int32_t q = s.qc[u];
          keep[w] &= (q != c4[w].x) & (q != c4[w].y) & (q != c4[w].z) & (q != c4[w].w);
        }
    } else {
#pragma unroll
      for (int w = 0; w < kWalk; ++w) {
        if (keep[w] && tt[w] > 0) {
          const int32_t* jc = kcodes + (static_cast<int64_t>(j[w]) * p.h_kv + h) * p.b;
          for (int y = 0; y < p.b; ++y) {
            const int32_t c = jc[y];
            for (int u = 0; u < tt[w]; ++u) keep[w] &= (s.qc[u] != c);
          }
        }
      }
    }
#pragma unroll
    for (int w = 0; w < kWalk; ++w) {
      const unsigned bal = __ballot_sync(0xffffffffu, keep[w]);
      const int slot = count + __popc(bal & ((1u << lane) - 1u));
      if (keep[w] && slot < CAP) jlist[slot] = j[w];
      count += __popc(bal);
    }
    if (count > CAP) break;                     // overflows this tier: no need to walk further
  }
  if (count > CAP || k_eff > kMaxSel) {
    if (lane == 0) out_list[atomicAdd(out_count, 1)] = static_cast<int32_t>(unit);
    return;
  }
  __syncwarp();

  // ---- 2. score the kept keys, 32 per batch, on tensor cores ----
  const T* kbase = static_cast<const T*>(p.k) + bat * p.k_sb + static_cast<int64_t>(h) * p.k_sh;
  for (int b0 = 0; b0 < count; b0 += kBatch) {
    uint4 kr[4][KSTEPS / 2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {           // lane (gid, tig): key b0+8nt+gid, dims 32kp+8tig..+7
      const int c = b0 + nt * 8 + gid;
      const int32_t jj = jlist[c < count ? c : b0];
      const T* row = kbase + static_cast<int64_t>(jj) * p.k_sn + 8 * tig;
#pragma unroll
      for (int kp = 0; kp < KSTEPS / 2; ++kp) kr[nt][kp] = __ldg(reinterpret_cast<const uint4*>(row + kp * 32));
    }
    float sc[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < KSTEPS / 2; ++kp) {
        mma16816<T>(sc[nt], qa[2 * kp], kr[nt][kp].x, kr[nt][kp].y);
        mma16816<T>(sc[nt], qa[2 * kp + 1], kr[nt][kp].z, kr[nt][kp].w);
      }
    }
    if (gid == 0) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = b0 + nt * 8 + 2 * tig + e;
          if (c < count)
            s.keys[c] = rank_key(sc[nt][e] + sc[nt][2 + e], static_cast<uint32_t>(jlist[c]));
        }
      }
    }
  }
  __syncwarp();

  // ---- 3. keep the top k: radix select over the 64-bit keys ----
  const int64_t obase = ((static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h) * p.top_k;
  const uint64_t* src = s.keys;
  int nsel = count;
  if (count > k_eff) {
    uint64_t prefix = 0ull, mask = 0ull;
    int need = k_eff;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int b = lane; b < 256; b += kWarp) hist[b] = 0u;
      __syncwarp();
      for (int idx = lane; idx < count; idx += kWarp) {
        const uint64_t kv = s.keys[idx];
        if ((kv & mask) == prefix) atomicAdd(&hist[(kv >> shift) & 255u], 1u);
      }
      __syncwarp();
      // lane l owns digits 255-8l .. 248-8l (descending)
      uint32_t cnt[8];
      uint32_t local = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        cnt[q] = hist[255 - 8 * lane - q];
        local += cnt[q];
      }
      uint32_t inc = local;
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      const uint32_t exc = inc - local;
      const bool mine = exc < static_cast<uint32_t>(need) && static_cast<uint32_t>(need) <= inc;
      int dsel = 0;
      uint32_t above = 0, dcount = 0;
      if (mine) {
        uint32_t acc = exc;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          if (dcount == 0 && acc + cnt[q] >= static_cast<uint32_t>(need)) {
            dsel = 255 - 8 * lane - q;
            above = acc;
            dcount = cnt[q];
          }
          acc += cnt[q];
        }
      }
      const int src_lane = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
      dsel = __shfl_sync(0xffffffffu, dsel, src_lane);
      above = __shfl_sync(0xffffffffu, above, src_lane);
      dcount = __shfl_sync(0xffffffffu, dcount, src_lane);
      prefix |= static_cast<uint64_t>(dsel) << shift;
      mask |= 0xffull << shift;
      need -= static_cast<int>(above);
      if (dcount == static_cast<uint32_t>(need)) break;
      __syncwarp();
    }
    // compact the keys >= prefix (exactly k_eff of them) into sel[]
    int base = 0;
    for (int idx0 = 0; idx0 < count; idx0 += kWarp) {
      const int idx = idx0 + lane;
      const uint64_t kv = idx < count ? s.keys[idx] : 0ull;
      const bool take = idx < count && kv >= prefix;
      const unsigned bal = __ballot_sync(0xffffffffu, take);
      if (take) s.sel[base + __popc(bal & ((1u << lane) - 1u))] = kv;
      base += __popc(bal);
    }
    __syncwarp();
    src = s.sel;
    nsel = k_eff;
  }

  // ---- 4. sort the selected keys, write them; filler; padding ----
  // the network for the smallest power of two >= nsel (4 keys a lane for the
  // early queries of a causal head, which have few candidates)
  if (nsel <= 32 * 4) sort_and_write<4>(src, nsel, lane, p, obase);
  else if (nsel <= 32 * 8) sort_and_write<8>(src, nsel, lane, p, obase);
  else sort_and_write<16>(src, nsel, lane, p, obase);
  auto put = [&](int slot, int32_t jj) {
    if (p.index_i64) static_cast<int64_t*>(p.out)[obase + slot] = jj;
    else static_cast<int32_t*>(p.out)[obase + slot] = jj;
  };
  if (count < k_eff) {
    const int need = k_eff - count;
    const int words = (k_eff + 31) / 32;
    if (lane < words) s.bitmap[lane] = 0u;
    __syncwarp();
    for (int e = lane; e < count; e += kWarp) {
      const uint32_t jj = rank_key_index(s.keys[e]);
      if (jj < static_cast<uint32_t>(k_eff)) atomicOr(&s.bitmap[jj >> 5], 1u << (jj & 31));
    }
    __syncwarp();
    // the lowest `need` free indices, in order: 32 indices per step, ranked
    // by a ballot (coalesced stores; the loop ends once `need` are placed)
    int base = 0;
#pragma unroll 1
    for (int w0 = 0; w0 < k_eff && base < need; w0 += kWarp) {
      const int jj = w0 + lane;
      const bool fr = jj < k_eff && !((s.bitmap[jj >> 5] >> (jj & 31)) & 1u);
      const unsigned bal = __ballot_sync(0xffffffffu, fr);
      const int rank = base + __popc(bal & ((1u << lane) - 1u));
      if (fr && rank < need) put(count + rank, jj);
      base += __popc(bal);
    }
  }
  for (int e = k_eff + lane; e < p.top_k; e += kWarp) put(e, 0);
  if (p.cand_counts && lane == 0)
    p.cand_counts[(static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h] = count;
}

// All units (LIST false) or the units of a list (count read on the device;
// each warp claims the next unclaimed unit through a counter).  Register caps:
// six CTAs of the first tier per SM (8.5 KB of shared memory per warp; the
// few bytes it spills cost less than the warps gained), four of the second.
template <typename T, int D, int CAP, int UNITS, bool LIST>
__global__ void __launch_bounds__(UNITS * kWarp, LIST ? 4 : 6) rescore_mma_kernel(RescoreParams p, const int32_t* in_list,
                                                                    const int32_t* in_count, int32_t* in_next,
                                                                    int32_t* out_list, int32_t* out_count) {
  extern __shared__ __align__(128) unsigned char dyn[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  RsMmaSmem<CAP>& s = reinterpret_cast<RsMmaSmem<CAP>*>(dyn)[warp];
  const int64_t wi = static_cast<int64_t>(blockIdx.x) * UNITS + warp;
  if constexpr (!LIST) {
    // the tier1_rows lowest positions of every (bat, h): unit numbers
    // bh * n_q + [n_q - tier1_rows, n_q) (positions descend within a head)
    const int rows = p.tier1_rows;
    const int64_t units = static_cast<int64_t>(p.batch) * p.h_kv * rows;
    if (wi < units) {
      const int w = static_cast<int>(wi), bh = w / rows;        // unit numbers fit 32 bits (list entries)
      const int unit = rows == p.n_q ? w : bh * p.n_q + (p.n_q - rows) + (w - bh * rows);
      rescore_mma_unit<T, D, CAP>(p, unit, s, lane, out_list, out_count);
    }
  } else {
    // units differ in cost by several times: each warp claims the next unit
    // of the list when it is free (a fixed stride leaves the launch waiting
    // on the warps that drew the heaviest units)
    const int n = *in_count;
    while (true) {
      int it = 0;
      if (lane == 0) it = atomicAdd(in_next, 1);
      it = __shfl_sync(0xffffffffu, it, 0);
      if (it >= n) break;
      rescore_mma_unit<T, D, CAP>(p, in_list[it], s, lane, out_list, out_count);
      __syncwarp();
    }
  }
}

bool rescore_mma_supported(const RescoreParams& p, ssa_dtype dt) {
  return (dt == SSA_BF16 || dt == SSA_F16) && (p.d == 64 || p.d == 128) && p.a <= 32;
}

// The units that start in the second tier, [bh * n_q, bh * n_q + rows) for
// every (bat, h), as its first list entries.
__global__ void rescore_prefill_kernel(int32_t* list, int32_t* count, int64_t heads, int n_q, int rows) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = heads * rows;
  if (t < total) list[t] = static_cast<int32_t>((t / rows) * n_q + t % rows);
  if (t == 0) *count = static_cast<int32_t>(total);
}

// Query rows (per (bat, h), counted from the lowest position) that start in
// the first tier.  With uniformly used codes a query at position pos has
// about a * b * (pos + 1) / n_codes candidates under the causal mask
// (a * b * n / n_codes without it); a query expected to hold more than 1.25
// times the first tier's room would nearly always overflow it after walking
// that many entries, so it starts in the second tier.  Any split gives the
// same results: every tier computes the same function of a unit.
static int tier1_rows(const RescoreParams& p, int cap1) {
  const double per_key = static_cast<double>(p.a) * p.b / p.n_codes;
  const double limit = 1.25 * cap1;
  if (!p.causal) return per_key * p.n > limit ? 0 : p.n_q;
  const double first_pos = std::ceil(limit / per_key);      // expected count above limit from here on
  // rows whose position lies below first_pos (positions ascend with the row)
  int rows = 0;
  for (int s = 0; s < p.seg.count; ++s) {
    const double below = first_pos - p.seg.pos[s];
    const int len = p.seg.row[s + 1] - p.seg.row[s];
    rows += below <= 0 ? 0 : (below >= len ? len : static_cast<int>(below));
  }
  return rows;
}

// A persistent launch of a list tier: as many CTAs per SM as fit.
template <typename Kern>
static cudaError_t launch_list_tier(Kern kern, int warps, size_t smem, const RescoreParams& p, const int32_t* in_list,
                                    const int32_t* in_count, int32_t* in_next, int32_t* out_list,
                                    int32_t* out_count, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, warps * kWarp, smem);
  if (e != cudaSuccess) return e;
  kern<<<static_cast<unsigned>(sms * (per_sm > 0 ? per_sm : 1)), warps * kWarp, smem, st>>>(
      p, in_list, in_count, in_next, out_list, out_count);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t launch_mma_t(const RescoreParams& p, cudaStream_t st) {
  for (int32_t* z : {p.ovf2_count, p.ovf2_next, p.ovf3_count, p.ovf3_next}) {
    const cudaError_t e = cudaMemsetAsync(z, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return e;
  }
  // tier 1: room for 512 candidates, all units but those expected to need
  // more (which go to tier 2's list first); overflow -> tier 2's list
  constexpr int U1 = SSA_RS_UNITS, C1 = 512;
  RescoreParams p1 = p;
  p1.tier1_rows = tier1_rows(p, C1);
  const int64_t heads = static_cast<int64_t>(p.batch) * p.h_kv;
  cudaError_t e = cudaSuccess;
  if (p1.tier1_rows < p.n_q) {
    const int64_t pre = heads * (p.n_q - p1.tier1_rows);
    rescore_prefill_kernel<<<static_cast<unsigned>(cdiv(pre, 256)), 256, 0, st>>>(p.ovf2_list, p.ovf2_count, heads,
                                                                                p.n_q, p.n_q - p1.tier1_rows);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (p1.tier1_rows > 0) {
    const size_t smem1 = sizeof(RsMmaSmem<C1>) * U1;
    auto k1 = rescore_mma_kernel<T, D, C1, U1, false>;
    e = cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem1));
    if (e != cudaSuccess) return e;
    const int64_t units1 = heads * p1.tier1_rows;
    k1<<<static_cast<unsigned>(cdiv(units1, U1)), U1 * kWarp, smem1, st>>>(p1, nullptr, nullptr, nullptr,
                                                                          p.ovf2_list, p.ovf2_count);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  // tier 2: room for 1024 (4 warps per CTA, warps claiming units from the
  // list); overflow -> tier 3
  constexpr int U2 = 4, C2 = 1024;
  e = launch_list_tier(rescore_mma_kernel<T, D, C2, U2, true>, U2, sizeof(RsMmaSmem<C2>) * U2, p, p.ovf2_list,
                       p.ovf2_count, p.ovf2_next, p.ovf3_list, p.ovf3_count, st);
  if (e != cudaSuccess) return e;
  // tier 3: room for 2048 (2 warps per CTA, 25 KB of shared memory a warp);
  // overflow -> the CTA-wide path
  constexpr int U3 = 2, C3 = 2048;
  return launch_list_tier(rescore_mma_kernel<T, D, C3, U3, true>, U3, sizeof(RsMmaSmem<C3>) * U3, p, p.ovf3_list,
                          p.ovf3_count, p.ovf3_next, p.ovf_list, p.ovf_count, st);
}

cudaError_t launch_rescore_mma(const RescoreParams& p, ssa_dtype dt, cudaStream_t st) {
  if (dt == SSA_BF16) return p.d == 64 ? launch_mma_t<__nv_bfloat16, 64>(p, st) : launch_mma_t<__nv_bfloat16, 128>(p, st);
  return p.d == 64 ? launch_mma_t<__half, 64>(p, st) : launch_mma_t<__half, 128>(p, st);
}

}  // namespace ssa
