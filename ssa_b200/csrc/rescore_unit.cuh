// Per-unit pieces of the candidate re-score (stage 2) shared by the kernel
// that walks each query's buckets (rescore_mma.cu) and the bucket-major path
// (rescore_bucket.cu): the shared-memory layout of a unit, the group-mean
// query, the top-k selection, the sort and the output.  Both paths compute a
// unit's scores with the same tensor-core fragments and these functions, so
// their outputs agree bit for bit.
#pragma once

#include <climits>

#include "common.cuh"
#include "kernels.cuh"
#include "mma_utils.cuh"

namespace ssa {

constexpr int kMaxSel = 512;        // k handled on this path

// SEL: room for the selected keys -- k at most; at least CAP/2 where the
// walking kernel keeps its CAP kept key indices there, at least 128 for the
// histogram.
template <int CAP, int SEL = (CAP / 2 > kMaxSel ? CAP / 2 : kMaxSel)>
struct __align__(128) RsMmaSmem {
  static_assert(SEL >= 128, "the radix histogram takes the last 1 KB of sel");
  uint64_t keys[CAP];                          // ranking keys of all candidates
  // kept key indices (CAP int32), then the selected keys (k <= SEL)
  // (its last 1 KB doubles as the radix-select histogram, and before the walk
  // as the group-mean query: neither overlaps a live use of sel)
  uint64_t sel[SEL];
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
// stage (not per element) and every compare-exchange is one compare and two
// selects.  The stage loops from k2 = 2E on stay rolled (run-time distances):
// the whole network is a few hundred instructions of code, so the warps of a
// CTA do not evict one another's instructions.
template <typename K, int E>
__device__ __forceinline__ void cx_desc(K (&key)[E], int e, int f, bool desc) {
  const K x = key[e], y = key[f];
  const bool sw = (x > y) != desc;           // equal keys: either order
  key[e] = sw ? y : x;
  key[f] = sw ? x : y;
}

template <typename K, int E>
__device__ __forceinline__ void sort_desc_blocked(K (&key)[E], int lane) {
  constexpr int N = 32 * E;
  // k2 < E: within each lane, direction fixed by e
#pragma unroll
  for (int k2 = 2; k2 < E; k2 <<= 1)
#pragma unroll
    for (int jj = k2 >> 1; jj > 0; jj >>= 1)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if ((e ^ jj) > e) cx_desc<K, E>(key, e, e ^ jj, (e & k2) == 0);
  // k2 = E: each lane's E keys in the direction of the lane's parity
  {
    const bool desc = (lane & 1) == 0;
#pragma unroll
    for (int jj = E >> 1; jj > 0; jj >>= 1)
#pragma unroll
      for (int e = 0; e < E; ++e)
        if ((e ^ jj) > e) cx_desc<K, E>(key, e, e ^ jj, desc);
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
        const K other = __shfl_xor_sync(0xffffffffu, key[e], j / E);
        key[e] = ((key[e] > other) == keep_max) ? key[e] : other;
      }
    }
#pragma unroll
    for (int jj = E >> 1; jj > 0; jj >>= 1)        // partner in the same lane
#pragma unroll
      for (int e = 0; e < E; ++e)
        if ((e ^ jj) > e) cx_desc<K, E>(key, e, e ^ jj, desc);
  }
}

// Sort the nsel keys at src (shared memory, any order) descending and write
// their indices in order at out[obase ..].  The network runs on 32-bit keys:
// the top bits of each 64-bit ranking key (its score) with the key's slot in
// src below them, so every compare-exchange is one 32-bit compare and every
// shuffle one word.  The full keys are then fetched by slot; keys whose top
// bits are equal form runs in arbitrary order, which an odd-even
// transposition pass over the full keys puts in order (one or two rounds;
// it stops when a round swaps nothing, and 32*E rounds sort any input).
template <int E>
__device__ __forceinline__ void sort_and_write(const uint64_t* src, int nsel, int lane, const RescoreParams& p,
                                               int64_t obase) {
  constexpr int SB = E <= 8 ? 8 : 9;          // bits of a slot number: 32 * E <= 2^SB
  constexpr uint32_t kSlot = (1u << SB) - 1u;
  static_assert(32 * E <= (1 << SB) && E % 2 == 0 && E >= 4, "slot bits");
  uint32_t k32[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {              // any input order: read conflict-free
    const int idx = e * 32 + lane;
    k32[e] = idx < nsel ? ((static_cast<uint32_t>(src[idx] >> 32) & ~kSlot) | static_cast<uint32_t>(idx)) : 0u;
  }
  // real keys have a nonzero high word (a float's order key), so padding sorts last
  sort_desc_blocked<uint32_t, E>(k32, lane);
  uint64_t key[E];
#pragma unroll
  for (int e = 0; e < E; ++e) key[e] = lane * E + e < nsel ? src[k32[e] & kSlot] : 0ull;
#pragma unroll 1
  for (int round = 0; round < 32 * E; ++round) {
    bool sw = false;
#pragma unroll
    for (int e = 0; e + 1 < E; e += 2)        // pairs (2m, 2m+1): inside the lane
      if (key[e] < key[e + 1]) {
        const uint64_t t = key[e]; key[e] = key[e + 1]; key[e + 1] = t; sw = true;
      }
#pragma unroll
    for (int e = 1; e + 1 < E; e += 2)        // pairs (2m+1, 2m+2) inside the lane ...
      if (key[e] < key[e + 1]) {
        const uint64_t t = key[e]; key[e] = key[e + 1]; key[e + 1] = t; sw = true;
      }
    // ... and across lanes: this lane's last key and the next lane's first
    const uint64_t next = __shfl_down_sync(0xffffffffu, key[0], 1);
    const uint64_t prev = __shfl_up_sync(0xffffffffu, key[E - 1], 1);
    const bool give = lane < kWarp - 1 && key[E - 1] < next;
    const bool take = lane > 0 && prev < key[0];
    if (give) key[E - 1] = next;
    if (take) key[0] = prev;
    if (!__any_sync(0xffffffffu, sw || give || take)) break;
  }
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

// The group-mean query of unit (bat, i, h), mean over the g query heads of
// KV head h (ssa/router.py:180-191), in fp32 into qs[0 .. D): the heads are
// summed in one fixed order (lane l holds 8-dim chunk l % (D/8) of heads
// l / (D/8), l / (D/8) + 32 / (D/8), ...; the chunk sums meet through xor
// shuffles), so every kernel that calls this gets the same bits.
template <typename T, int D>
__device__ __forceinline__ void group_mean_smem(const RescoreParams& p, int bat, int i, int h, int lane, float* qs) {
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
  if (lane < CH) {
    const float inv_g = 1.0f / static_cast<float>(p.group);
#pragma unroll
    for (int u = 0; u < 8; ++u) qs[ch * 8 + u] = p.group != 1 ? x[u] * inv_g : x[u];
  }
  __syncwarp();
}

// Steps 3 and 4 of a unit: keep the top k of its `count` candidates (a warp
// radix select, 8 bits per pass over the 64-bit ranking keys), sort them,
// write them in order at out[row * top_k ..], then the filler and the zero
// padding, and the candidate count.  `keys[0 .. entries)` holds the
// candidates' ranking keys, either in shared memory (entries == count, the
// form every path uses when the candidates fit) or in global memory, where
// entries may also hold zeros (empty slots, below every real key) -- the
// global form is used only when count > k, so a zero is never selected and no
// filler is needed.  The result does not depend on the order of the keys.
template <int CAP, int SEL>
__device__ __forceinline__ void select_sort_write(const RescoreParams& p, RsMmaSmem<CAP, SEL>& s, const uint64_t* keys,
                                                  int entries, int count, int k_eff, int lane, int64_t row) {
  uint32_t* hist = reinterpret_cast<uint32_t*>(s.sel) + (sizeof(s.sel) / 4 - 256);
  const int64_t obase = row * p.top_k;
  // ---- 3. keep the top k: radix select over the 64-bit keys ----
  const uint64_t* src = keys;
  int nsel = count;
  if (count > k_eff) {
    uint64_t prefix = 0ull, mask = 0ull;
    int need = k_eff;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int b = lane; b < 256; b += kWarp) hist[b] = 0u;
      __syncwarp();
      for (int idx = lane; idx < entries; idx += kWarp) {
        const uint64_t kv = keys[idx];
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
    for (int idx0 = 0; idx0 < entries; idx0 += kWarp) {
      const int idx = idx0 + lane;
      const uint64_t kv = idx < entries ? keys[idx] : 0ull;
      const bool take = idx < entries && kv >= prefix;
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
      const uint32_t jj = rank_key_index(keys[e]);
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
    p.cand_counts[row] = count;
}

}  // namespace ssa
