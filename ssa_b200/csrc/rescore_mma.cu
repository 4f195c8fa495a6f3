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
// (long sequences only) start in the second tier.  Where the bucket-major path
// (rescore_bucket.cu) applies it replaces the first tier: the units it has no
// buffer room for start in the second.  The per-unit pieces both paths share
// are in rescore_unit.cuh.
#include <cmath>

#include "rescore_unit.cuh"

namespace ssa {

#ifndef SSA_RS_UNITS
#define SSA_RS_UNITS 4
#endif
constexpr int kBatch = 32;          // candidates per MMA batch (4 n-tiles)
constexpr int kWalk = 4;            // bucket-walk iterations whose loads are issued together

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
    float* qs = reinterpret_cast<float*>(hist);      // D floats; sel is free until the walk
    group_mean_smem<T, D>(p, bat, i, h, lane, qs);
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

  select_sort_write(p, s, s.keys, count, count, k_eff, lane,
                         (static_cast<int64_t>(bat) * p.n_q + i) * p.h_kv + h);
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

// Tier 1 of the walking kernel: room for 512 candidates, all units but those
// expected to need more (which go to tier 2's list first); overflow -> tier
// 2's list.
template <typename T, int D>
static cudaError_t launch_tier1(const RescoreParams& p, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  constexpr int U1 = SSA_RS_UNITS, C1 = 512;
  RescoreParams p1 = p;
  p1.tier1_rows = tier1_rows(p, C1);
  const int64_t heads = static_cast<int64_t>(p.batch) * p.h_kv;
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
  return cudaSuccess;
}

template <typename T, int D>
static cudaError_t launch_mma_t(const RescoreParams& p, cudaStream_t st) {
  for (int32_t* z : {p.ovf2_count, p.ovf2_next, p.ovf3_count, p.ovf3_next}) {
    const cudaError_t e = cudaMemsetAsync(z, 0, sizeof(int32_t), st);
    if (e != cudaSuccess) return e;
  }
  cudaError_t e = cudaSuccess;
  if (p.qbar) {
    // the bucket-major path takes every unit it has room for; the rest go
    // to tier 2's list
    e = launch_rescore_bucket<T, D>(p, st);
    if (e != cudaSuccess) return e;
  } else {
    e = launch_tier1<T, D>(p, st);
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
