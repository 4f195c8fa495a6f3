// K4 for 16-bit inputs on tensor cores: sparse exact attention with the
// selected keys on the M axis of m16n8k16 MMAs.
//
// Reference: sparse_exact_attention, ssa/attention.py:12-115 (with the
// per-KV-head gather k[idx, h]; `scale` divides the logits).
//
// One warp per (bat, i, h) unit.  Its k selected keys are processed in chunks
// of 16: the chunk's K and V rows are gathered with 16-byte cp.async into a
// per-warp shared-memory ring (rows XOR-swizzled in 16-byte units so that
// ldmatrix reads are conflict-free), overlapping the next chunk's gather with
// the current chunk's math.  The g query heads of the KV group are the N
// columns (one tile of 8 heads for g <= 8, two for g <= 16):
//   S^T = K Q^T  : A = the chunk's 16 K rows (ldmatrix), B = Q^T (registers)
//   online softmax in fp32 per head column (exp2 form; a head's reference max
//   moves only when it grows by more than 2^8)
//   O^T += V^T P^T: A = V^T (ldmatrix.trans), B = P^T taken from the S^T
//                 fragments by one movmatrix.trans per 8x8 block, as a hi + lo
//                 pair of 16-bit operands (two MMAs) so that the probabilities
//                 keep ~16 significant bits
// With keys on M, a chunk costs d/16 * NT MMAs for S and 2 * d/16 * NT for
// P.V, and a lane holds 4 scores per head tile.
// Units are ordered head-major (all queries of one (bat, h) before the next),
// so the K/V rows of the heads in flight stay resident in L2.
#include "common.cuh"
#include "kernels.cuh"
#include "mma_utils.cuh"

namespace ssa {

#ifndef SSA_ATTN_WARPS
#define SSA_ATTN_WARPS 1
#endif
#ifndef SSA_ATTN_STAGES
#define SSA_ATTN_STAGES 2
#endif
constexpr int kMmaWarps = SSA_ATTN_WARPS;     // warps (units) per CTA
constexpr int kStages = SSA_ATTN_STAGES;      // chunks of 16 keys per warp ring
constexpr int kChunk = 16;

// byte offset of 16-byte segment `seg` of row `row` in a [kChunk][D] tile
template <int D>
__device__ __forceinline__ uint32_t swz(int row, int seg) {
  return static_cast<uint32_t>(row * (D * 2) + ((seg ^ (row & 7)) << 4));
}

template <typename T, int D, int NT>
__global__ void __launch_bounds__(kMmaWarps * kWarp) sparse_attn_mma_kernel(AttnParams p) {
  constexpr int SEGS = D * 2 / 16;                // 16-byte segments per row
  constexpr int TILE = kChunk * D * 2;            // bytes of one K (or V) chunk
  constexpr int KSTEPS = D / 16;                  // k-steps of S^T, m-tiles of O^T
  constexpr int ROWS = kWarp / SEGS;              // rows one pass of the warp copies
  constexpr int PASSES = kChunk / ROWS;
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const uint32_t wbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem + warp * (2 * kStages * TILE)));

  const int64_t units = static_cast<int64_t>(p.batch) * p.h_kv * p.n_q;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kMmaWarps + warp;
  if (unit >= units) return;
  const int64_t bh = unit / p.n_q;                // head-major order
  const int i = static_cast<int>(unit % p.n_q);
  const int h = static_cast<int>(bh % p.h_kv);
  const int64_t bat = bh / p.h_kv;
  const int g = p.group;
  const int gid = lane >> 2, tig = lane & 3;

  const char* kb = reinterpret_cast<const char*>(static_cast<const T*>(p.k) + bat * p.k_sb +
                                                 static_cast<int64_t>(h) * p.k_sh);
  const char* vb = reinterpret_cast<const char*>(static_cast<const T*>(p.v) + bat * p.v_sb +
                                                 static_cast<int64_t>(h) * p.v_sh);
  const uint32_t ksn = static_cast<uint32_t>(p.k_sn * 2), vsn = static_cast<uint32_t>(p.v_sn * 2);
  const char* ib = static_cast<const char*>(p.idx) +
                   (bat * p.i_sb + static_cast<int64_t>(i) * p.i_sn + static_cast<int64_t>(h) * p.i_sh) *
                       (p.index_i64 ? 8 : 4);
  const int64_t limit = seg_pos(p.seg, i);

  // ---- Q^T as the B operand: column n = head 8 nt + gid, k = head dims ----
  uint32_t qb[NT][KSTEPS][2];
  {
    const T* qrow = static_cast<const T*>(p.q) + bat * p.q_sb + static_cast<int64_t>(i) * p.q_sn +
                    static_cast<int64_t>(h) * g * p.q_sh;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int head = nt * 8 + gid;
      const bool ok = head < g;
      const uint32_t* qr = reinterpret_cast<const uint32_t*>(qrow + static_cast<int64_t>(ok ? head : 0) * p.q_sh);
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        qb[nt][ks][0] = ok ? __ldg(qr + ks * 8 + tig) : 0u;
        qb[nt][ks][1] = ok ? __ldg(qr + ks * 8 + 4 + tig) : 0u;
      }
    }
  }

  // ---- chunk gather ----
  const int nchunks = (p.top_k + kChunk - 1) / kChunk;
  // Lanes 0..15 read index slot c*16 + lane (-1 past k).  The value is used
  // one chunk later (prep), so the load's latency hides behind a chunk of math.
  auto load_index = [&](int c) -> int64_t {
    const int kk = c * kChunk + lane;
    if (lane >= kChunk || c >= nchunks || kk >= p.top_k) return -1;
    return p.index_i64 ? reinterpret_cast<const int64_t*>(ib)[kk]
                       : static_cast<int64_t>(reinterpret_cast<const int32_t*>(ib)[kk]);
  };
  // Returns the lane's key clamped into [0, n) (an out-of-range index is
  // flagged and masked) and the chunk's valid mask.
  auto prep = [&](int c, int64_t jj, uint32_t& vm) -> int {
    const int kk = c * kChunk + lane;
    int j = 0;
    bool valid = false;
    if (lane < kChunk && kk < p.top_k) {
      if (jj < 0 || jj >= p.n) {
        set_status(p.status, SSA_DEVICE_INDEX_OOB);
      } else {
        j = static_cast<int>(jj);
        valid = !p.causal || jj <= limit;
      }
    }
    vm = __ballot_sync(0xffffffffu, valid) & 0xffffu;
    return j;
  };
  const int crow = lane / SEGS, cseg = lane % SEGS;
  auto issue = [&](int stage, int jl) {
    const uint32_t kdst = wbase + stage * (2 * TILE);
    const uint32_t vdst = kdst + TILE;
#pragma unroll
    for (int t = 0; t < PASSES; ++t) {
      const int row = t * ROWS + crow;
      const uint32_t j = static_cast<uint32_t>(__shfl_sync(0xffffffffu, jl, row));
      cp_async16(kdst + swz<D>(row, cseg), kb + static_cast<uint64_t>(j) * ksn + cseg * 16);
      cp_async16(vdst + swz<D>(row, cseg), vb + static_cast<uint64_t>(j) * vsn + cseg * 16);
    }
    cp_commit();
  };

  float o[KSTEPS][NT][4];
#pragma unroll
  for (int mt = 0; mt < KSTEPS; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
  float m[NT][2], l[NT][2];                       // heads 8nt + 2tig + e: reference max, partial sum
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) m[nt][0] = m[nt][1] = -INFINITY, l[nt][0] = l[nt][1] = 0.f;
  const float sl2 = p.inv_scale * 1.4426950408889634f;

  // ring of kStages chunks: chunk c lives in stage c % kStages; one cp.async
  // group per chunk (empty groups past the end keep wait_group constant);
  // vq holds the valid masks of the chunks in flight, jpre the raw index of
  // the next chunk to issue
  uint32_t vq[kStages];
#pragma unroll
  for (int sidx = 0; sidx < kStages - 1; ++sidx) {
    vq[sidx] = 0u;
    if (sidx < nchunks) issue(sidx, prep(sidx, load_index(sidx), vq[sidx]));
    else cp_commit();
  }
  int64_t jpre = load_index(kStages - 1);
  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % kStages;
    const int nx = c + kStages - 1;
    vq[kStages - 1] = 0u;
    if (nx < nchunks) issue(nx % kStages, prep(nx, jpre, vq[kStages - 1]));
    else cp_commit();
    jpre = load_index(nx + 1);
    const uint32_t vmask = vq[0];
#pragma unroll
    for (int q = 0; q + 1 < kStages; ++q) vq[q] = vq[q + 1];
    cp_wait<kStages - 1>();
    __syncwarp();

    const uint32_t kt = wbase + stage * (2 * TILE);
    const uint32_t vt = kt + TILE;
    // ---- S^T = K Q^T : rows = keys gid / gid+8, columns = heads; even and
    // odd k-steps accumulate separately (two independent MMA chains) ----
    float s[NT][4], s2[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = s2[nt][e] = 0.f;
    {
      const int mi = lane >> 3, r = lane & 7;
      const int row = (mi & 1) * 8 + r;
#pragma unroll
      for (int ks = 0; ks < KSTEPS; ++ks) {
        // matrices: (keys 0-7, dims 16ks..+7), (keys 8-15, ..), (keys 0-7, +8..15), (keys 8-15, +8..15)
        uint32_t a[4];
        ldsm_x4(kt + swz<D>(row, ks * 2 + (mi >> 1)), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<T>((ks & 1) ? s2[nt] : s[nt], a, qb[nt][ks][0], qb[nt][ks][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) s[nt][e] += s2[nt][e];
    }
    // ---- online softmax per head column ----
    const bool ok0 = (vmask >> gid) & 1u, ok1 = (vmask >> (gid + 8)) & 1u;
    uint32_t bh[NT][2], bl[NT][2];                // P^T fragments (hi, lo) for keys 0-7 / 8-15
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float x[4];
      x[0] = ok0 ? s[nt][0] * sl2 : -INFINITY;
      x[1] = ok0 ? s[nt][1] * sl2 : -INFINITY;
      x[2] = ok1 ? s[nt][2] * sl2 : -INFINITY;
      x[3] = ok1 ? s[nt][3] * sl2 : -INFINITY;
      float pr[4];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float hm = fmaxf(x[e], x[2 + e]);
        hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, 4));
        hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, 8));
        hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, 16));
        // Lazy rescaling: the reference point of a head moves only when the
        // chunk max exceeds it by more than 2^8, so P stays <= 256 and O, l
        // are rescaled rarely.  The lanes of one head take the same branch.
        if (hm > m[nt][e] + 8.f) {
          const float al = m[nt][e] == -INFINITY ? 0.f : ex2_approx(m[nt][e] - hm);
          l[nt][e] *= al;
#pragma unroll
          for (int mt = 0; mt < KSTEPS; ++mt) { o[mt][nt][e] *= al; o[mt][nt][2 + e] *= al; }
          m[nt][e] = hm;
        }
        const float mr = m[nt][e];
        pr[e] = mr == -INFINITY ? 0.f : ex2_approx(x[e] - mr);
        pr[2 + e] = mr == -INFINITY ? 0.f : ex2_approx(x[2 + e] - mr);
        l[nt][e] += pr[e] + pr[2 + e];
      }
      uint32_t h0, l0, h1, l1;
      split2<T>(pr[0], pr[1], h0, l0);            // [key gid][heads 2tig, 2tig+1]
      split2<T>(pr[2], pr[3], h1, l1);            // [key gid+8][..]
      bh[nt][0] = movm_t(h0);                     // [head gid][keys 2tig, 2tig+1]
      bh[nt][1] = movm_t(h1);
      bl[nt][0] = movm_t(l0);
      bl[nt][1] = movm_t(l1);
    }
    // ---- O^T += V^T P^T ----
    {
      const int mi = lane >> 3, r = lane & 7;
      const int row = (mi >> 1) * 8 + r;
#pragma unroll
      for (int mt = 0; mt < KSTEPS; ++mt) {
        // matrices: (keys 0-7, dims 16mt..+7), (keys 0-7, +8..15), (keys 8-15, ..), (keys 8-15, +8..15)
        uint32_t a[4];
        ldsm_x4_t(vt + swz<D>(row, mt * 2 + (mi & 1)), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816<T>(o[mt][nt], a, bh[nt][0], bh[nt][1]);
          mma16816<T>(o[mt][nt], a, bl[nt][0], bl[nt][1]);
        }
      }
    }
    __syncwarp();
  }
  // ---- normalise, transpose back to [head][dims] and store heads < g ----
  T* orow = static_cast<T*>(p.out) + bat * p.o_sb + static_cast<int64_t>(i) * p.o_sn +
            static_cast<int64_t>(h) * g * p.o_sh;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float inv[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float t = l[nt][e];
      t += __shfl_xor_sync(0xffffffffu, t, 4);
      t += __shfl_xor_sync(0xffffffffu, t, 8);
      t += __shfl_xor_sync(0xffffffffu, t, 16);
      // a head with no valid key (every index masked) has t = 0 and o = 0:
      // its output row is written as zeros
      inv[e] = t > 0.f ? 1.0f / t : 0.f;
    }
    const int head = nt * 8 + gid;
    uint32_t* dst = reinterpret_cast<uint32_t*>(orow + static_cast<int64_t>(head < g ? head : 0) * p.o_sh);
#pragma unroll
    for (int mt = 0; mt < KSTEPS; ++mt) {
      const uint32_t w0 = movm_t(pack2<T>(o[mt][nt][0] * inv[0], o[mt][nt][1] * inv[1]));
      const uint32_t w1 = movm_t(pack2<T>(o[mt][nt][2] * inv[0], o[mt][nt][3] * inv[1]));
      if (head < g) {
        dst[mt * 8 + tig] = w0;                   // dims 16mt + 2tig, +1
        dst[mt * 8 + 4 + tig] = w1;               // dims 16mt + 8 + 2tig, +1
      }
    }
  }
}

bool sparse_attn_mma_supported(const AttnParams& p, ssa_dtype dt) {
  const auto al = [](const void* x, uintptr_t a) { return (reinterpret_cast<uintptr_t>(x) % a) == 0; };
  // row strides of K and V in bytes must fit the kernel's 32-bit row offsets
  const bool rows32 = p.k_sn >= 0 && p.v_sn >= 0 && p.k_sn * 2 <= INT32_MAX && p.v_sn * 2 <= INT32_MAX &&
                      static_cast<int64_t>(p.n) * p.k_sn * 2 < (int64_t(1) << 32) &&
                      static_cast<int64_t>(p.n) * p.v_sn * 2 < (int64_t(1) << 32);
  return (dt == SSA_BF16 || dt == SSA_F16) && (p.d == 64 || p.d == 128) && p.group <= 16 && rows32 &&
         al(p.q, 4) && al(p.out, 4) && al(p.v, 16) && al(p.k, 16) &&
         (p.q_sn % 2 == 0) && (p.q_sh % 2 == 0) && (p.q_sb % 2 == 0) && (p.o_sn % 2 == 0) &&
         (p.o_sh % 2 == 0) && (p.o_sb % 2 == 0) && (p.v_sn % 8 == 0) && (p.v_sh % 8 == 0) &&
         (p.v_sb % 8 == 0);
}

template <typename T, int D>
static cudaError_t launch_mma(const AttnParams& p, cudaStream_t st) {
  const int64_t units = static_cast<int64_t>(p.batch) * p.h_kv * p.n_q;
  const unsigned blocks = static_cast<unsigned>(cdiv(units, kMmaWarps));
  const size_t smem = static_cast<size_t>(kMmaWarps) * 2 * kStages * kChunk * D * 2;
  auto kern = p.group <= 8 ? sparse_attn_mma_kernel<T, D, 1> : sparse_attn_mma_kernel<T, D, 2>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  kern<<<blocks, kMmaWarps * kWarp, smem, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_sparse_attn_mma(const AttnParams& p, ssa_dtype dt, cudaStream_t st) {
  if (dt == SSA_BF16) return p.d == 64 ? launch_mma<__nv_bfloat16, 64>(p, st) : launch_mma<__nv_bfloat16, 128>(p, st);
  return p.d == 64 ? launch_mma<__half, 64>(p, st) : launch_mma<__half, 128>(p, st);
}

}  // namespace ssa
