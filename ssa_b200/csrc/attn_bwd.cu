// Backward of K4 (sparse exact attention): dQ, dK, dV for
//   out[i, hq] = sum_t P[i, hq, t] v[idx[i, h, t], h],
//   P[i, hq, :] = softmax_t( q[i, hq] . k[idx[i, h, t], h] / scale ),
// hq in the GQA group of KV head h, causal slots (idx > q_offset + i) masked.
// The reference differentiates its gather/einsum forward with autograd
// (ssa/attention.py:93-113, exercised by tests/test_integration.py:32-49);
// the per-slot semantics match: a key selected twice counts twice.
//
// One warp per (bat, i, h) unit, lanes over the head dimension (d/32 values
// each).  The unit's g query rows, their output gradients and the dQ
// accumulators sit in shared memory.  Pass 1 recomputes each head's logit
// maximum and softmax sum over the k slots; pass 2 revisits the slots:
//   dP = dO . v_j,  dS = P (dP - Delta),  Delta = dO . out,
//   dQ += dS k_j / scale,  dK[j] += sum_g dS q_g / scale,  dV[j] += sum_g P dO_g.
// dK and dV go to fp32 buffers with atomic adds (several queries select the
// same key), so their rounding depends on the order the adds land in.
#include "common.cuh"
#include "kernels.cuh"

namespace ssa {

constexpr int kBwdMaxG = 16;

__device__ __forceinline__ float bwd_warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename T, int DPL>
__global__ void __launch_bounds__(kWarp) sparse_attn_bwd_kernel(AttnBwdParams p) {
  extern __shared__ __align__(16) float sm[];
  const AttnParams& a = p.fwd;
  const int g = a.group, d = a.d;
  float* qs = sm;                         // [g][d]  q
  float* dos = qs + kBwdMaxG * d;         // [g][d]  dO
  float* dqs = dos + kBwdMaxG * d;        // [g][d]  dQ accumulators
  const int lane = threadIdx.x;
  const int64_t unit = blockIdx.x;
  const int bh = static_cast<int>(unit / a.n_q);
  const int i = static_cast<int>(unit % a.n_q);
  const int bat = bh / a.h_kv, h = bh % a.h_kv;

  const T* qrow = static_cast<const T*>(a.q) + bat * a.q_sb + static_cast<int64_t>(i) * a.q_sn +
                  static_cast<int64_t>(h) * g * a.q_sh;
  const T* orow = static_cast<const T*>(a.out) + bat * a.o_sb + static_cast<int64_t>(i) * a.o_sn +
                  static_cast<int64_t>(h) * g * a.o_sh;
  const T* gorow = static_cast<const T*>(p.d_out) + bat * a.o_sb + static_cast<int64_t>(i) * a.o_sn +
                   static_cast<int64_t>(h) * g * a.o_sh;
  float delta[kBwdMaxG];
#pragma unroll
  for (int gg = 0; gg < kBwdMaxG; ++gg) {
    float part = 0.f;
    if (gg < g) {
      for (int e = lane; e < d; e += kWarp) {
        const float qv = Elem<T>::to_f(qrow[gg * a.q_sh + e]);
        const float go = Elem<T>::to_f(gorow[gg * a.o_sh + e]);
        qs[gg * d + e] = qv;
        dos[gg * d + e] = go;
        dqs[gg * d + e] = 0.f;
        part += go * Elem<T>::to_f(orow[gg * a.o_sh + e]);
      }
    }
    delta[gg] = bwd_warp_sum(part);
  }
  __syncwarp();

  const T* kb = static_cast<const T*>(a.k) + bat * a.k_sb + static_cast<int64_t>(h) * a.k_sh;
  const T* vb = static_cast<const T*>(a.v) + bat * a.v_sb + static_cast<int64_t>(h) * a.v_sh;
  const char* ib = static_cast<const char*>(a.idx) +
                   (bat * a.i_sb + static_cast<int64_t>(i) * a.i_sn + static_cast<int64_t>(h) * a.i_sh) *
                       (a.index_i64 ? 8 : 4);
  const int64_t limit = seg_pos(a.seg, i);
  auto slot_key = [&](int t, bool& valid) -> int64_t {
    const int64_t j = a.index_i64 ? reinterpret_cast<const int64_t*>(ib)[t]
                                  : static_cast<int64_t>(reinterpret_cast<const int32_t*>(ib)[t]);
    valid = j >= 0 && j < a.n && (!a.causal || j <= limit);
    return j;
  };
  // logits of all g heads for key row kr (lane's dims)
  auto logits = [&](const float (&kr)[DPL], float (&s)[kBwdMaxG]) {
#pragma unroll
    for (int gg = 0; gg < kBwdMaxG; ++gg) {
      float part = 0.f;
      if (gg < g) {
#pragma unroll
        for (int u = 0; u < DPL; ++u) {
          const int e = lane + u * kWarp;
          if (e < d) part += qs[gg * d + e] * kr[u];
        }
      }
      s[gg] = bwd_warp_sum(part) * a.inv_scale;
    }
  };
  auto load_row = [&](const T* base, int64_t j, int64_t sn, float (&r)[DPL]) {
#pragma unroll
    for (int u = 0; u < DPL; ++u) {
      const int e = lane + u * kWarp;
      r[u] = e < d ? Elem<T>::to_f(base[j * sn + e]) : 0.f;
    }
  };

  // ---- pass 1: per-head maximum and softmax sum ----
  float m[kBwdMaxG], l[kBwdMaxG];
#pragma unroll
  for (int gg = 0; gg < kBwdMaxG; ++gg) { m[gg] = -INFINITY; l[gg] = 0.f; }
  for (int t = 0; t < a.top_k; ++t) {
    bool valid;
    const int64_t j = slot_key(t, valid);
    if (!valid) {
      if (j < 0 || j >= a.n) set_status(a.status, SSA_DEVICE_INDEX_OOB);
      continue;
    }
    float kr[DPL], s[kBwdMaxG];
    load_row(kb, j, a.k_sn, kr);
    logits(kr, s);
#pragma unroll
    for (int gg = 0; gg < kBwdMaxG; ++gg) {
      if (s[gg] > m[gg]) {
        l[gg] = l[gg] * expf(m[gg] - s[gg]) + 1.f;
        m[gg] = s[gg];
      } else {
        l[gg] += expf(s[gg] - m[gg]);
      }
    }
  }

  // ---- pass 2: gradients ----
  for (int t = 0; t < a.top_k; ++t) {
    bool valid;
    const int64_t j = slot_key(t, valid);
    if (!valid) continue;
    float kr[DPL], vr[DPL], s[kBwdMaxG];
    load_row(kb, j, a.k_sn, kr);
    load_row(vb, j, a.v_sn, vr);
    logits(kr, s);
    float pr[kBwdMaxG], ds[kBwdMaxG];
#pragma unroll
    for (int gg = 0; gg < kBwdMaxG; ++gg) {
      float part = 0.f;
      if (gg < g) {
#pragma unroll
        for (int u = 0; u < DPL; ++u) {
          const int e = lane + u * kWarp;
          if (e < d) part += dos[gg * d + e] * vr[u];
        }
      }
      const float dp = bwd_warp_sum(part);
      pr[gg] = gg < g ? expf(s[gg] - m[gg]) / l[gg] : 0.f;
      ds[gg] = pr[gg] * (dp - delta[gg]);
    }
    float* dk = p.d_k + (static_cast<int64_t>(bat) * a.n + j) * p.acc_sn + static_cast<int64_t>(h) * d;
    float* dv = p.d_v + (static_cast<int64_t>(bat) * a.n + j) * p.acc_sn + static_cast<int64_t>(h) * d;
#pragma unroll
    for (int u = 0; u < DPL; ++u) {
      const int e = lane + u * kWarp;
      if (e < d) {
        float gk = 0.f, gv = 0.f;
#pragma unroll
        for (int gg = 0; gg < kBwdMaxG; ++gg) {
          if (gg < g) {
            dqs[gg * d + e] += ds[gg] * kr[u];
            gk += ds[gg] * qs[gg * d + e];
            gv += pr[gg] * dos[gg * d + e];
          }
        }
        atomicAdd(dk + e, gk * a.inv_scale);
        atomicAdd(dv + e, gv);
      }
    }
  }
  __syncwarp();
  T* dqrow = static_cast<T*>(p.d_q) + bat * a.q_sb + static_cast<int64_t>(i) * a.q_sn +
             static_cast<int64_t>(h) * g * a.q_sh;
  for (int gg = 0; gg < g; ++gg)
    for (int e = lane; e < d; e += kWarp) dqrow[gg * a.q_sh + e] = Elem<T>::from_f(dqs[gg * d + e] * a.inv_scale);
}

template <typename T>
static cudaError_t launch_bwd_t(const AttnBwdParams& p, cudaStream_t st) {
  const int64_t units = static_cast<int64_t>(p.fwd.batch) * p.fwd.h_kv * p.fwd.n_q;
  if (units == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(3) * kBwdMaxG * p.fwd.d * sizeof(float);
  const unsigned blocks = static_cast<unsigned>(units);
#define SSA_BWD(DPL)                                                                            \
  do {                                                                                          \
    auto kern = sparse_attn_bwd_kernel<T, DPL>;                                                 \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e != cudaSuccess) return e;                                                             \
    kern<<<blocks, kWarp, smem, st>>>(p);                                                       \
  } while (0)
  const int dpl = static_cast<int>(cdiv(p.fwd.d, kWarp));
  if (dpl <= 2) SSA_BWD(2);
  else if (dpl <= 4) SSA_BWD(4);
  else SSA_BWD(8);
#undef SSA_BWD
  return cudaGetLastError();
}

cudaError_t launch_sparse_attn_bwd(const AttnBwdParams& p, ssa_dtype dt, cudaStream_t st) {
  if (dt == SSA_F32) return launch_bwd_t<float>(p, st);
  if (dt == SSA_BF16) return launch_bwd_t<__nv_bfloat16>(p, st);
  return launch_bwd_t<__half>(p, st);
}

}  // namespace ssa
