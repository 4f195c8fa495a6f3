// K4 for 16-bit inputs on tensor cores: sparse exact attention with the
// g query heads of a KV group as the M rows of m16n8k16 MMAs.
//
// Reference: sparse_exact_attention, ssa/attention.py:12-115 (with the
// per-KV-head gather k[idx, h]; `scale` divides the logits).
//
// One warp per (bat, i, h) unit.  Its k selected keys are processed in chunks
// of 16: the chunk's K and V rows are gathered with 16-byte cp.async into a
// per-warp two-stage shared-memory ring (rows XOR-swizzled in 16-byte units
// so that ldmatrix reads are conflict-free), overlapping the next chunk's
// gather with the current chunk's math.
//   S = Q K^T   : A = Q (16 x d; rows >= g are zero), B = K rows via ldmatrix
//   online softmax in fp32 on the accumulator fragments (exp2 form, with the
//   reference max moved only when it grows by more than 2^8)
//   O += P V    : A = P re-packed from the S fragments as a hi + lo pair of
//                 16-bit operands (two MMAs), B = V via ldmatrix.trans
// Units are ordered head-major (all queries of one (bat, h) before the next),
// so the K/V rows of the heads in flight stay resident in L2.
#include "common.cuh"
#include "kernels.cuh"
#include "mma_utils.cuh"

namespace ssa {

#ifndef SSA_ATTN_WARPS
#define SSA_ATTN_WARPS 4
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

template <typename T, int D>
__global__ void __launch_bounds__(kMmaWarps * kWarp) sparse_attn_mma_kernel(AttnParams p) {
  constexpr int SEGS = D * 2 / 16;                // 16-byte segments per row
  constexpr int TILE = kChunk * D * 2;            // bytes of one K (or V) chunk
  constexpr int KSTEPS = D / 16;                  // QK k-steps
  constexpr int NT = D / 8;                       // PV n-tiles
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  unsigned char* wbuf = smem + warp * (2 * kStages * TILE);  // [stage][K|V][TILE]
  const uint32_t wbase = static_cast<uint32_t>(__cvta_generic_to_shared(wbuf));

  const int64_t units = static_cast<int64_t>(p.batch) * p.h_kv * p.n_q;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kMmaWarps + warp;
  if (unit >= units) return;
  const int64_t bh = unit / p.n_q;                // head-major order
  const int i = static_cast<int>(unit % p.n_q);
  const int h = static_cast<int>(bh % p.h_kv);
  const int64_t bat = bh / p.h_kv;
  const int g = p.group;
  const int gid = lane >> 2, tig = lane & 3;

  const T* kb = static_cast<const T*>(p.k) + bat * p.k_sb + static_cast<int64_t>(h) * p.k_sh;
  const T* vb = static_cast<const T*>(p.v) + bat * p.v_sb + static_cast<int64_t>(h) * p.v_sh;
  const char* ib = static_cast<const char*>(p.idx) +
                   (bat * p.i_sb + static_cast<int64_t>(i) * p.i_sn + static_cast<int64_t>(h) * p.i_sh) *
                       (p.index_i64 ? 8 : 4);
  const int64_t limit = static_cast<int64_t>(p.q_offset) + i;

  // ---- Q fragments (A operand), rows = query heads of the group ----
  uint32_t qa[KSTEPS][4];
  {
    const T* qrow = static_cast<const T*>(p.q) + bat * p.q_sb + static_cast<int64_t>(i) * p.q_sn +
                    static_cast<int64_t>(h) * g * p.q_sh;
    const bool r0 = gid < g, r1 = gid + 8 < g;
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(qrow + static_cast<int64_t>(gid) * p.q_sh);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(qrow + static_cast<int64_t>(gid + 8) * p.q_sh);
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      const int c = ks * 8 + tig;                  // 32-bit column (pairs of elements)
      qa[ks][0] = r0 ? __ldg(q0 + c) : 0u;
      qa[ks][1] = r1 ? __ldg(q1 + c) : 0u;
      qa[ks][2] = r0 ? __ldg(q0 + c + 4) : 0u;
      qa[ks][3] = r1 ? __ldg(q1 + c + 4) : 0u;
    }
  }

  // ---- chunk gather: lane handles segment (lane % SEGS') of rows ----
  const int nchunks = (p.top_k + kChunk - 1) / kChunk;
  auto load_index = [&](int c) -> int64_t {    // lanes 0..15: key of slot c*16 + lane (or -1)
    const int kk = c * kChunk + (lane & 15);
    int64_t j = -1;
    if (kk < p.top_k) {
      j = p.index_i64 ? reinterpret_cast<const int64_t*>(ib)[kk]
                      : static_cast<int64_t>(reinterpret_cast<const int32_t*>(ib)[kk]);
    }
    return j;
  };
  auto issue = [&](int c, int stage, int64_t jl) {
    // jl: this lane's key (lanes 0..15 meaningful); row r's key comes from lane r
    const uint32_t kdst = wbase + stage * (2 * TILE);
    const uint32_t vdst = kdst + TILE;
#pragma unroll
    for (int t = 0; t < kChunk * SEGS / kWarp; ++t) {
      const int s = t * kWarp + lane;
      const int row = s / SEGS, seg = s % SEGS;
      int64_t j = __shfl_sync(0xffffffffu, jl, row);
      if (j < 0 || j >= p.n) j = 0;                // masked below; keep the copy in bounds
      cp_async16(kdst + swz<D>(row, seg), kb + j * p.k_sn + seg * 8);
      cp_async16(vdst + swz<D>(row, seg), vb + j * p.v_sn + seg * 8);
    }
    cp_commit();
  };

  float o[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY;           // reference max, rows gid / gid+8 (log2 units)
  float l0 = 0.f, l1 = 0.f;                       // this thread's partial row sums
  const float sl2 = p.inv_scale * 1.4426950408889634f;

  // ring of kStages chunks: chunk c lives in stage c % kStages; one cp.async
  // group per chunk (empty groups past the end keep wait_group constant)
  int64_t jring[kStages];
#pragma unroll
  for (int sidx = 0; sidx < kStages - 1; ++sidx) {
    jring[sidx] = sidx < nchunks ? load_index(sidx) : -1;
    if (sidx < nchunks) issue(sidx, sidx, jring[sidx]);
    else cp_commit();
  }
  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % kStages;
    const int nx = c + kStages - 1;
    if (nx < nchunks) {
      jring[nx % kStages] = load_index(nx);
      issue(nx, nx % kStages, jring[nx % kStages]);
    } else {
      cp_commit();
    }
    cp_wait<kStages - 1>();
    __syncwarp();
    const int64_t j_cur = jring[stage];
    // validity of the chunk's 16 keys
    bool valid = false;
    if (lane < kChunk) {
      const int kk = c * kChunk + lane;
      if (kk < p.top_k) {
        if (j_cur < 0 || j_cur >= p.n) set_status(p.status, SSA_DEVICE_INDEX_OOB);
        else valid = !p.causal || j_cur <= limit;
      }
    }
    const uint32_t vmask = __ballot_sync(0xffffffffu, valid) & 0xffffu;

    const uint32_t kt = wbase + stage * (2 * TILE);
    const uint32_t vt = kt + TILE;
    // ---- S = Q K^T : two n-tiles of 8 keys ----
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) {
      // matrices: (keys 0-7, dims ks*16..+7), (keys 0-7, +8..15), (keys 8-15, ..), (keys 8-15, +8..)
      const int mi = lane >> 3, r = lane & 7;
      const int row = (mi >> 1) * 8 + r;
      const int seg = ks * 2 + (mi & 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kt + swz<D>(row, seg), b0, b1, b2, b3);
      mma16816<T>(s[0], qa[ks], b0, b1);
      mma16816<T>(s[1], qa[ks], b2, b3);
    }
    // ---- online softmax (rows gid: c0,c1 ; gid+8: c2,c3) ----
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = nt * 8 + tig * 2 + e;
        const bool ok = (vmask >> key) & 1u;
        s[nt][e] = ok ? s[nt][e] * sl2 : -INFINITY;
        s[nt][2 + e] = ok ? s[nt][2 + e] * sl2 : -INFINITY;
        mx0 = fmaxf(mx0, s[nt][e]);
        mx1 = fmaxf(mx1, s[nt][2 + e]);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // Lazy rescaling: the reference point m of a row moves only when the chunk
    // max exceeds it by more than 2^8, so P stays <= 256 and O, l are rescaled
    // rarely.  Both quad lanes of a row take the same branch.
    if (mx0 > m0 + 8.f) {
      const float a0 = m0 == -INFINITY ? 0.f : exp2f(m0 - mx0);
      l0 *= a0;
#pragma unroll
      for (int t = 0; t < NT; ++t) { o[t][0] *= a0; o[t][1] *= a0; }
      m0 = mx0;
    }
    if (mx1 > m1 + 8.f) {
      const float a1 = m1 == -INFINITY ? 0.f : exp2f(m1 - mx1);
      l1 *= a1;
#pragma unroll
      for (int t = 0; t < NT; ++t) { o[t][2] *= a1; o[t][3] *= a1; }
      m1 = mx1;
    }
    float pr[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pr[nt][e] = m0 == -INFINITY ? 0.f : exp2f(s[nt][e] - m0);
        pr[nt][2 + e] = m1 == -INFINITY ? 0.f : exp2f(s[nt][2 + e] - m1);
      }
    }
    l0 += pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l1 += pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
    // ---- O += P V, with P = P_hi + P_lo split into two 16-bit operands so that
    // the probabilities keep ~16 significant bits ----
    uint32_t pa[4], pb[4];
    split2<T>(pr[0][0], pr[0][1], pa[0], pb[0]);
    split2<T>(pr[0][2], pr[0][3], pa[1], pb[1]);
    split2<T>(pr[1][0], pr[1][1], pa[2], pb[2]);
    split2<T>(pr[1][2], pr[1][3], pa[3], pb[3]);
#pragma unroll
    for (int t2 = 0; t2 < NT / 2; ++t2) {
      // matrices: (keys 0-7, dims t2*16..+7), (keys 8-15, same), (keys 0-7, +8..15), (keys 8-15, +8..15)
      const int mi = lane >> 3, r = lane & 7;
      const int row = (mi & 1) * 8 + r;
      const int seg = t2 * 2 + (mi >> 1);
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vt + swz<D>(row, seg), b0, b1, b2, b3);
      mma16816<T>(o[2 * t2], pa, b0, b1);
      mma16816<T>(o[2 * t2], pb, b0, b1);
      mma16816<T>(o[2 * t2 + 1], pa, b2, b3);
      mma16816<T>(o[2 * t2 + 1], pb, b2, b3);
    }
    __syncwarp();
  }
  // ---- normalise and store rows gid (< g) ----
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  T* orow = static_cast<T*>(p.out) + bat * p.o_sb + static_cast<int64_t>(i) * p.o_sn +
            static_cast<int64_t>(h) * g * p.o_sh;
  if (gid < g) {
    const float inv = 1.0f / l0;
    uint32_t* dst = reinterpret_cast<uint32_t*>(orow + static_cast<int64_t>(gid) * p.o_sh);
#pragma unroll
    for (int t = 0; t < NT; ++t) dst[t * 4 + tig] = pack2<T>(o[t][0] * inv, o[t][1] * inv);
  }
  if (gid + 8 < g) {
    const float inv = 1.0f / l1;
    uint32_t* dst = reinterpret_cast<uint32_t*>(orow + static_cast<int64_t>(gid + 8) * p.o_sh);
#pragma unroll
    for (int t = 0; t < NT; ++t) dst[t * 4 + tig] = pack2<T>(o[t][2] * inv, o[t][3] * inv);
  }
}

bool sparse_attn_mma_supported(const AttnParams& p, ssa_dtype dt) {
  const auto al = [](const void* x, uintptr_t a) { return (reinterpret_cast<uintptr_t>(x) % a) == 0; };
  return (dt == SSA_BF16 || dt == SSA_F16) && (p.d == 64 || p.d == 128) && p.group <= 16 &&
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
  auto kern = sparse_attn_mma_kernel<T, D>;
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
