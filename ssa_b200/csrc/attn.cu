// K4: sparse exact attention (stage 3).
//
// Reference: sparse_exact_attention, ssa/attention.py:12-115:
//   out[i, h*g+g'] = softmax_j( q[i,h*g+g'] . k[idx[i,h,j], h] / scale ) . v[idx[i,h,j], h]
// with `scale` a divisor (default sqrt(d), ssa/attention.py:37-38,107).  The
// reference's flattened gather picks the wrong rows for h_kv > 1
// (ssa/attention.py:76-91); this kernel gathers k[idx, h] / v[idx, h].
// With causal=1, keys j > q_offset + i are masked (-inf logit).  Duplicate
// indices count once per occurrence, as in the reference's gather.
//
// One warp per (bat, i, h) unit; the g query heads of the group share the
// unit's index list.  Keys are taken 32 at a time, one per lane, for the
// logits (the lane reads its key row with 16-byte loads); the online softmax
// runs in fp32; for P.V the chunk's probabilities are broadcast by shuffles
// and each lane accumulates its slice of the d output features from
// coalesced rows of V.
#include "common.cuh"
#include "kernels.cuh"

namespace ssa {

constexpr int kAttnWarps = 4;

template <typename T, int GMAX, int DPL>
__global__ void __launch_bounds__(kAttnWarps * kWarp) sparse_attn_kernel(AttnParams p) {
  extern __shared__ __align__(16) float qs_all[];   // [warps][GMAX][d] q * (1/scale)
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int bhs = p.batch * p.h_kv;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kAttnWarps + warp;
  const int64_t units = static_cast<int64_t>(p.n_q) * bhs;
  if (unit >= units) return;
  const int r = static_cast<int>(unit / p.n_q);          // head-major order
  const int i = static_cast<int>(unit % p.n_q);
  const int bat = r / p.h_kv, h = r % p.h_kv;
  const int d = p.d, g = p.group;
  float* qs = qs_all + static_cast<int64_t>(warp) * GMAX * d;
  const T* qrow = static_cast<const T*>(p.q) + bat * p.q_sb + static_cast<int64_t>(i) * p.q_sn +
                  static_cast<int64_t>(h) * g * p.q_sh;
  for (int gg = 0; gg < GMAX; ++gg)
    for (int e = lane; e < d; e += kWarp)
      qs[gg * d + e] = gg < g ? Elem<T>::to_f(qrow[gg * p.q_sh + e]) * p.inv_scale : 0.f;
  __syncwarp();

  const T* kb = static_cast<const T*>(p.k) + bat * p.k_sb + static_cast<int64_t>(h) * p.k_sh;
  const T* vb = static_cast<const T*>(p.v) + bat * p.v_sb + static_cast<int64_t>(h) * p.v_sh;
  const char* ib = static_cast<const char*>(p.idx) +
                   (bat * p.i_sb + static_cast<int64_t>(i) * p.i_sn + static_cast<int64_t>(h) * p.i_sh) *
                       (p.index_i64 ? 8 : 4);
  const int64_t limit = seg_pos(p.seg, i);
  constexpr float kLog2e = 1.4426950408889634f;

  float m_run[GMAX], l_lane[GMAX], o[GMAX][DPL];
#pragma unroll
  for (int gg = 0; gg < GMAX; ++gg) {
    m_run[gg] = -INFINITY;
    l_lane[gg] = 0.f;
#pragma unroll
    for (int t = 0; t < DPL; ++t) o[gg][t] = 0.f;
  }
  const int dim0 = lane * DPL;              // this lane's output features [dim0, dim0+DPL)
  const bool has_dims = dim0 < d;

  for (int c0 = 0; c0 < p.top_k; c0 += kWarp) {
    const int kk = c0 + lane;
    int64_t j = -1;
    bool valid = false;
    if (kk < p.top_k) {
      j = p.index_i64 ? reinterpret_cast<const int64_t*>(ib)[kk]
                      : static_cast<int64_t>(reinterpret_cast<const int32_t*>(ib)[kk]);
      if (j < 0 || j >= p.n) {
        set_status(p.status, SSA_DEVICE_INDEX_OOB);
      } else {
        valid = !p.causal || j <= limit;
      }
    }
    float sc[GMAX];
#pragma unroll
    for (int gg = 0; gg < GMAX; ++gg) sc[gg] = 0.f;
    if (valid) {
      const T* krow = kb + j * p.k_sn;
      for (int e = 0; e < d; e += 8) {
        float f[8];
        load8<T>(krow + e, f);
#pragma unroll
        for (int gg = 0; gg < GMAX; ++gg) {
          const float4 q0 = *reinterpret_cast<const float4*>(qs + gg * d + e);
          const float4 q1 = *reinterpret_cast<const float4*>(qs + gg * d + e + 4);
          float acc = sc[gg];
          acc = fmaf(f[0], q0.x, acc); acc = fmaf(f[1], q0.y, acc);
          acc = fmaf(f[2], q0.z, acc); acc = fmaf(f[3], q0.w, acc);
          acc = fmaf(f[4], q1.x, acc); acc = fmaf(f[5], q1.y, acc);
          acc = fmaf(f[6], q1.z, acc); acc = fmaf(f[7], q1.w, acc);
          sc[gg] = acc;
        }
      }
    }
    float pr[GMAX];
#pragma unroll
    for (int gg = 0; gg < GMAX; ++gg) {
      float s = valid ? sc[gg] : -INFINITY;
      float mx = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_run[gg], mx);
      if (m_new == -INFINITY) { pr[gg] = 0.f; continue; }   // nothing valid yet (warp-uniform)
      const float alpha = exp2f((m_run[gg] - m_new) * kLog2e);
      pr[gg] = valid ? exp2f((s - m_new) * kLog2e) : 0.f;
      l_lane[gg] = l_lane[gg] * alpha + pr[gg];
#pragma unroll
      for (int t = 0; t < DPL; ++t) o[gg][t] *= alpha;
      m_run[gg] = m_new;
    }
    const unsigned vmask = __ballot_sync(0xffffffffu, valid);
    unsigned rem = vmask;
    while (rem) {
      const int src = __ffs(rem) - 1;
      rem &= rem - 1;
      const int64_t jj = __shfl_sync(0xffffffffu, j, src);
      float pk[GMAX];
#pragma unroll
      for (int gg = 0; gg < GMAX; ++gg) pk[gg] = __shfl_sync(0xffffffffu, pr[gg], src);
      if (has_dims) {
        const T* vrow = vb + jj * p.v_sn + dim0;
        float vv[DPL];
#pragma unroll
        for (int t = 0; t < DPL; ++t) vv[t] = Elem<T>::to_f(vrow[t]);
#pragma unroll
        for (int gg = 0; gg < GMAX; ++gg)
#pragma unroll
          for (int t = 0; t < DPL; ++t) o[gg][t] = fmaf(pk[gg], vv[t], o[gg][t]);
      }
    }
  }
  T* orow = static_cast<T*>(p.out) + bat * p.o_sb + static_cast<int64_t>(i) * p.o_sn +
            static_cast<int64_t>(h) * g * p.o_sh;
#pragma unroll
  for (int gg = 0; gg < GMAX; ++gg) {
    float l = l_lane[gg];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (gg < g && has_dims) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;   // no valid key: a zero row
#pragma unroll
      for (int t = 0; t < DPL; ++t)
        if (dim0 + t < d) orow[gg * p.o_sh + dim0 + t] = Elem<T>::from_f(o[gg][t] * inv);
    }
  }
}

template <typename T, int GMAX>
static cudaError_t launch_attn_g(const AttnParams& p, cudaStream_t st) {
  const int64_t units = static_cast<int64_t>(p.n_q) * p.batch * p.h_kv;
  const unsigned blocks = static_cast<unsigned>(cdiv(units, kAttnWarps));
  const size_t smem = static_cast<size_t>(kAttnWarps) * GMAX * p.d * sizeof(float);
#define SSA_AT(DPL)                                                                        \
  do {                                                                                     \
    auto kern = sparse_attn_kernel<T, GMAX, DPL>;                                          \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    kern<<<blocks, kAttnWarps * kWarp, smem, st>>>(p);                                     \
  } while (0)
  if (p.d <= 32) SSA_AT(1);
  else if (p.d <= 64) SSA_AT(2);
  else if (p.d <= 128) SSA_AT(4);
  else SSA_AT(8);
#undef SSA_AT
  return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_attn_t(const AttnParams& p, cudaStream_t st) {
  if (p.group <= 1) return launch_attn_g<T, 1>(p, st);
  if (p.group <= 2) return launch_attn_g<T, 2>(p, st);
  if (p.group <= 4) return launch_attn_g<T, 4>(p, st);
  if (p.group <= 8) return launch_attn_g<T, 8>(p, st);
  return launch_attn_g<T, 16>(p, st);
}

cudaError_t launch_sparse_attn(const AttnParams& p, ssa_dtype dt, cudaStream_t st) {
  if (static_cast<int64_t>(p.n_q) * p.batch * p.h_kv == 0) return cudaSuccess;
  if (sparse_attn_mma_supported(p, dt)) return launch_sparse_attn_mma(p, dt, st);
  if (dt == SSA_F32) return launch_attn_t<float>(p, st);
  if (dt == SSA_BF16) return launch_attn_t<__nv_bfloat16>(p, st);
  return launch_attn_t<__half>(p, st);
}

}  // namespace ssa
