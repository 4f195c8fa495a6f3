// Stage 1 of the SSA router: routing projection, codebook scoring and the
// fused top-a (queries) / top-b (keys) code selection.
//
// Reference: CodebookRouter.forward, ssa/router.py:102-141, and
// get_code_assignment, ssa/router.py:261-275.
//
//   q_route[i,h] = normalize( W_qr . mean_g q[i, h*g+g'] )      [d_s]
//   k_route[j,h] = normalize( W_kr . k[j, h] )                  [d_s]
//   score[r, c]  = (route[r] . normalize(codebook[h, c])) / temperature
//   codes[r]     = top-a (queries) / top-b (keys) of score[r, :]
//
// The reference projects each query head and then averages over the GQA
// group (ssa/router.py:102-112); projecting the group mean is the same
// linear map, evaluated with g times fewer multiply-adds.
#include "common.cuh"
#include "kernels.cuh"
#include "mma_utils.cuh"

namespace ssa {

// ---------------------------------------------------------------------------
// K0: routing projection + L2 normalisation, in tiles of 64 rows.
//   1. all threads load the tile's rows with 16-byte loads and form the GQA
//      group mean in fp32 (shared memory, [64][d]);
//   2. warp w computes rows 8w..8w+7: lane c owns route component c (and
//      c + 32 when d_s = 64); W^T[e][c] comes from shared memory
//      (consecutive lanes, conflict-free) and x[row][e..e+3] is a broadcast
//      128-bit read, so 12 shared loads feed 32 FMAs;
//   3. each row is normalised by a warp reduction of its squares.
// Per output the FMA chain runs over e in increasing order, as a plain dot
// product would.
// ---------------------------------------------------------------------------
constexpr int kRpRows = 64;        // rows per tile
constexpr int kRpThreads = 256;    // 8 warps x 8 rows

// 8 consecutive elements as raw 16-byte words (two for fp32), converted later
// so that several loads can be in flight before the first is used.
template <typename T> struct Raw8 { uint4 a; };
template <> struct Raw8<float> { uint4 a, b; };
template <typename T>
__device__ __forceinline__ void raw8_load(const T* p, Raw8<T>& r) { r.a = __ldg(reinterpret_cast<const uint4*>(p)); }
template <>
__device__ __forceinline__ void raw8_load<float>(const float* p, Raw8<float>& r) {
  r.a = __ldg(reinterpret_cast<const uint4*>(p));
  r.b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
}
template <typename T>
__device__ __forceinline__ void raw8_zero(Raw8<T>& r) { r.a = make_uint4(0u, 0u, 0u, 0u); }
template <>
__device__ __forceinline__ void raw8_zero<float>(Raw8<float>& r) { r.a = r.b = make_uint4(0u, 0u, 0u, 0u); }
__device__ __forceinline__ void raw8_add(const Raw8<float>& r, float (&x)[8]) {
  x[0] += __uint_as_float(r.a.x); x[1] += __uint_as_float(r.a.y);
  x[2] += __uint_as_float(r.a.z); x[3] += __uint_as_float(r.a.w);
  x[4] += __uint_as_float(r.b.x); x[5] += __uint_as_float(r.b.y);
  x[6] += __uint_as_float(r.b.z); x[7] += __uint_as_float(r.b.w);
}
__device__ __forceinline__ void raw8_add(const Raw8<__nv_bfloat16>& r, float (&x)[8]) {
  const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] += __uint_as_float(w[i] << 16);
    x[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void raw8_add(const Raw8<__half>& r, float (&x)[8]) {
  const uint32_t w[4] = {r.a.x, r.a.y, r.a.z, r.a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    x[2 * i] += t.x;
    x[2 * i + 1] += t.y;
  }
}

template <typename T, typename TW, bool TWO>
__global__ void __launch_bounds__(kRpThreads) route_project_kernel(RouteProjectParams p) {
  extern __shared__ __align__(16) float smem[];
  const int d = p.d, d_s = p.d_s;
  float* wt = smem;                          // [d][d_s]
  float* xs = smem + d * d_s;                // [kRpRows][d]
  const TW* w = static_cast<const TW*>(p.w);
  for (int t = threadIdx.x; t < d * d_s; t += blockDim.x) {
    const int e = t / d_s, c = t % d_s;      // w is [d_s][d]; consecutive t -> consecutive banks
    wt[t] = Elem<TW>::to_f(w[c * d + e]);
  }
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const T* src = static_cast<const T*>(p.x);
  const float inv_g = 1.0f / static_cast<float>(p.group);
  const int chunks = d / 8;
  const int items = kRpRows * chunks;
  const bool has0 = lane < d_s;
  for (int64_t tile0 = static_cast<int64_t>(blockIdx.x) * kRpRows; tile0 < p.rows;
       tile0 += static_cast<int64_t>(gridDim.x) * kRpRows) {
    __syncthreads();                         // W^T written; the previous tile's rows consumed
    // ---- 1. group means of the tile's rows: a thread takes two 8-element
    // items at a time and issues up to four heads' loads of both together ----
    for (int idx0 = threadIdx.x; idx0 < items; idx0 += 2 * kRpThreads) {
      const T* base[2];
      bool ok[2];
      float x[2][8];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int idx = idx0 + q * kRpThreads;
        const int rl = idx / chunks, ch = idx % chunks;
        const int64_t row = tile0 + rl;      // row = ((bat * h_kv + h) * n_rows + i)
        ok[q] = idx < items && row < p.rows;
        const int64_t i = row % p.n_rows;
        const int64_t bh = row / p.n_rows;
        const int h = static_cast<int>(bh % p.h_kv);
        const int64_t bat = bh / p.h_kv;
        base[q] = src + (ok[q] ? bat * p.stride_b + i * p.stride_n + static_cast<int64_t>(h) * p.group * p.stride_h +
                                     ch * 8
                               : 0);
#pragma unroll
        for (int u = 0; u < 8; ++u) x[q][u] = 0.f;
      }
      for (int g0 = 0; g0 < p.group; g0 += 4) {
        Raw8<T> r[2][4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            if (ok[q] && g0 + t < p.group) raw8_load<T>(base[q] + (g0 + t) * p.stride_h, r[q][t]);
            else raw8_zero<T>(r[q][t]);
          }
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int q = 0; q < 2; ++q)
            if (g0 + t < p.group) raw8_add(r[q][t], x[q]);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int idx = idx0 + q * kRpThreads;
        if (idx < items) {
          if (p.group != 1) {
#pragma unroll
            for (int u = 0; u < 8; ++u) x[q][u] *= inv_g;
          }
          const int rl = idx / chunks, ch = idx % chunks;
          float4* dst = reinterpret_cast<float4*>(xs + rl * d + ch * 8);
          dst[0] = make_float4(x[q][0], x[q][1], x[q][2], x[q][3]);
          dst[1] = make_float4(x[q][4], x[q][5], x[q][6], x[q][7]);
        }
      }
    }
    __syncthreads();
    // ---- 2. projection: rows r0..r0+7 of the tile ----
    const int r0 = warp * 8;
    float acc0[8], acc1[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) acc0[r] = acc1[r] = 0.f;
    for (int e = 0; e < d; e += 4) {
      float w0[4], w1[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        w0[u] = has0 ? wt[(e + u) * d_s + lane] : 0.f;
        if (TWO) w1[u] = wt[(e + u) * d_s + lane + kWarp];
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + (r0 + r) * d + e);
        acc0[r] = fmaf(w0[0], xv.x, acc0[r]);
        acc0[r] = fmaf(w0[1], xv.y, acc0[r]);
        acc0[r] = fmaf(w0[2], xv.z, acc0[r]);
        acc0[r] = fmaf(w0[3], xv.w, acc0[r]);
        if (TWO) {
          acc1[r] = fmaf(w1[0], xv.x, acc1[r]);
          acc1[r] = fmaf(w1[1], xv.y, acc1[r]);
          acc1[r] = fmaf(w1[2], xv.z, acc1[r]);
          acc1[r] = fmaf(w1[3], xv.w, acc1[r]);
        }
      }
    }
    // ---- 3. normalise and store ----
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float v0 = has0 ? acc0[r] : 0.f;
      const float v1 = TWO ? acc1[r] : 0.f;
      float ss = v0 * v0 + v1 * v1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float nrm = fmaxf(sqrtf(ss), 1e-12f);
      const int64_t row = tile0 + r0 + r;
      if (row < p.rows) {
        float* out = p.out + row * d_s;
        if (has0) out[lane] = v0 / nrm;
        if (TWO) out[lane + kWarp] = v1 / nrm;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// K0 on the tensor cores (16-bit inputs): route[r] = W . sum_g x[r, g] as an
// mma.sync m16n8k16 GEMM with K = g * d (the group's heads one after another,
// each against the same W) and N = d_s, then the 1/g scale and the L2
// normalisation in the epilogue.
//
// W (fp32, or 16-bit) is split into three 16-bit terms of the input's type,
// w = w0 + w1 + w2 exactly for bf16 (8 + 8 + 8 significant bits) and to
// below 2^-24 |w| for f16, and each A fragment is multiplied by all three:
// every product x * w is exact and only the fp32 accumulation rounds.
//
// K order: the dot product over e is order-free, so the k index of the MMA
// is mapped onto e to let each thread fill its A fragments with 16-byte loads
// straight from global memory: within a 32-element chunk c of a row, quad
// position p loads e in [32c + 8p, 32c + 8p + 8); k step 2c + h takes
// e = 32c + 8p + 4h + {0, 1} as fragment columns 2p, 2p + 1 and
// e = 32c + 8p + 4h + {2, 3} as columns 2p + 8, 2p + 9.  The W image in
// shared memory holds each thread's B fragments in that order,
// [k step][n tile][term][lane] x 8 bytes, so a warp reads 256 contiguous bytes
// per fragment (no bank conflicts).
//
// A warp owns 32 consecutive rows (two m tiles); rows are in (bat, h, i)
// order as in the FMA version.
// ---------------------------------------------------------------------------
constexpr int kRmWarps = 4;
constexpr int kRmMT = 2;           // m tiles (16 rows) per warp

// Rotate-half RoPE of 8 elements of the first half (lo) and their partners
// d/2 further on (hi), evaluated as the PyTorch expression
// x * cos + cat(-x2, x1) * sin in the 16-bit dtype T: each product and the sum
// rounded to T.
template <typename T>
__device__ __forceinline__ void rope8(uint4& lo, uint4& hi, const uint4 c_lo, const uint4 c_hi, const uint4 s_lo,
                                      const uint4 s_hi) {
  auto r = [](float x) { return Elem<T>::to_f(Elem<T>::from_f(x)); };
  auto unpack = [](const uint4 v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const T* h = reinterpret_cast<const T*>(&w[i]);
      f[2 * i] = Elem<T>::to_f(h[0]);
      f[2 * i + 1] = Elem<T>::to_f(h[1]);
    }
  };
  float a[8], b[8], cl[8], ch[8], sl[8], sh[8];
  unpack(lo, a); unpack(hi, b); unpack(c_lo, cl); unpack(c_hi, ch); unpack(s_lo, sl); unpack(s_hi, sh);
  uint32_t ol[4], oh[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float xl[2], xh[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int e = 2 * i + u;
      xl[u] = r(r(a[e] * cl[e]) + r(-b[e] * sl[e]));
      xh[u] = r(r(b[e] * ch[e]) + r(a[e] * sh[e]));
    }
    ol[i] = pack2<T>(xl[0], xl[1]);
    oh[i] = pack2<T>(xh[0], xh[1]);
  }
  lo = make_uint4(ol[0], ol[1], ol[2], ol[3]);
  hi = make_uint4(oh[0], oh[1], oh[2], oh[3]);
}

template <typename T, typename TW, int NT, bool ROPE>
__global__ void __launch_bounds__(kRmWarps * kWarp) route_project_mma_kernel(RouteProjectParams p) {
  extern __shared__ __align__(16) uint2 wimg[];          // [d/16][NT][3][32]
  const int d = p.d;
  const int ksteps = d / 16;
  const TW* w = static_cast<const TW*>(p.w);
  for (int t = threadIdx.x; t < ksteps * NT * kWarp; t += blockDim.x) {
    const int ln = t % kWarp, nt = (t / kWarp) % NT, s = t / (kWarp * NT);
    const int n = nt * 8 + ln / 4;
    const int e0 = 32 * (s / 2) + 8 * (ln % 4) + 4 * (s % 2);
    float x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) x[u] = Elem<TW>::to_f(w[static_cast<int64_t>(n) * d + e0 + u]);
#pragma unroll
    for (int term = 0; term < 3; ++term) {
      float tv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        tv[u] = Elem<T>::to_f(Elem<T>::from_f(x[u]));     // this term
        x[u] -= tv[u];                                    // what the next terms carry
      }
      wimg[((s * NT + nt) * 3 + term) * kWarp + ln] = make_uint2(pack2<T>(tv[0], tv[1]), pack2<T>(tv[2], tv[3]));
    }
  }
  __syncthreads();

  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int gq = lane / 4, qp = lane % 4;
  const T* src = static_cast<const T*>(p.x);
  const float inv_g = 1.0f / static_cast<float>(p.group);
  const int64_t tasks = cdiv(p.rows, 16 * kRmMT);
  for (int64_t task = static_cast<int64_t>(blockIdx.x) * kRmWarps + warp; task < tasks;
       task += static_cast<int64_t>(gridDim.x) * kRmWarps) {
    // this thread's rows: m tile mt, half hh -> row task*32 + 16 mt + 8 hh + gq
    const T* base[kRmMT][2];
    int64_t tab[kRmMT][2], obase[kRmMT][2];      // RoPE table row and output row offsets
    bool ok[kRmMT][2];
#pragma unroll
    for (int mt = 0; mt < kRmMT; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int64_t row = task * (16 * kRmMT) + 16 * mt + 8 * hh + gq;
        ok[mt][hh] = row < p.rows;
        const int64_t rr = ok[mt][hh] ? row : 0;
        const int64_t i = rr % p.n_rows, bh = rr / p.n_rows;
        const int h = static_cast<int>(bh % p.h_kv);
        const int64_t bat = bh / p.h_kv;
        base[mt][hh] = src + bat * p.stride_b + i * p.stride_n + static_cast<int64_t>(h) * p.group * p.stride_h +
                       8 * qp;
        if constexpr (ROPE) {
          tab[mt][hh] = bat * p.rope_sb + (p.pos_offset + i) * p.rope_sn + 8 * qp;
          obase[mt][hh] = bat * p.out_sb + i * p.out_sn + static_cast<int64_t>(h) * p.group * p.out_sh + 8 * qp;
        }
      }
    float acc[kRmMT][NT][4];
#pragma unroll
    for (int mt = 0; mt < kRmMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[mt][nt][u] = 0.f;

    for (int gg = 0; gg < p.group; ++gg) {
      for (int c0 = 0; c0 < d / 32; c0 += 4) {
        // up to four 32-element chunks of every row in flight
        uint4 raw[4][kRmMT][2];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int mt = 0; mt < kRmMT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              raw[cc][mt][hh] = make_uint4(0u, 0u, 0u, 0u);
              if (ok[mt][hh] && c0 + cc < d / 32)
                raw[cc][mt][hh] = __ldg(reinterpret_cast<const uint4*>(
                    base[mt][hh] + static_cast<int64_t>(gg) * p.stride_h + 32 * (c0 + cc)));
            }
        if constexpr (ROPE) {
          // d is 64 or 128 here, so this pass holds every chunk of the rows:
          // chunk cc pairs with chunk cc + d/64 (elements e and e + d/2)
          const T* tcos = static_cast<const T*>(p.rope_cos);
          const T* tsin = static_cast<const T*>(p.rope_sin);
          T* xo = static_cast<T*>(p.x_out);
#pragma unroll
          for (int mt = 0; mt < kRmMT; ++mt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              if (!ok[mt][hh]) continue;
              const T* cr = tcos + tab[mt][hh];
              const T* sr = tsin + tab[mt][hh];
              T* orow = xo + obase[mt][hh] + static_cast<int64_t>(gg) * p.out_sh;
              auto pair = [&](uint4& lo, uint4& hi, int clo, int chi) {
                const uint4 c_lo = __ldg(reinterpret_cast<const uint4*>(cr + 32 * clo));
                const uint4 c_hi = __ldg(reinterpret_cast<const uint4*>(cr + 32 * chi));
                const uint4 s_lo = __ldg(reinterpret_cast<const uint4*>(sr + 32 * clo));
                const uint4 s_hi = __ldg(reinterpret_cast<const uint4*>(sr + 32 * chi));
                rope8<T>(lo, hi, c_lo, c_hi, s_lo, s_hi);
                *reinterpret_cast<uint4*>(orow + 32 * clo) = lo;
                *reinterpret_cast<uint4*>(orow + 32 * chi) = hi;
              };
              if (d == 128) {
                pair(raw[0][mt][hh], raw[2][mt][hh], 0, 2);
                pair(raw[1][mt][hh], raw[3][mt][hh], 1, 3);
              } else {
                pair(raw[0][mt][hh], raw[1][mt][hh], 0, 1);
              }
            }
        }
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          if (c0 + cc >= d / 32) break;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int s = 2 * (c0 + cc) + h2;
            uint32_t a[kRmMT][4];
#pragma unroll
            for (int mt = 0; mt < kRmMT; ++mt) {
              a[mt][0] = h2 ? raw[cc][mt][0].z : raw[cc][mt][0].x;
              a[mt][1] = h2 ? raw[cc][mt][1].z : raw[cc][mt][1].x;
              a[mt][2] = h2 ? raw[cc][mt][0].w : raw[cc][mt][0].y;
              a[mt][3] = h2 ? raw[cc][mt][1].w : raw[cc][mt][1].y;
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int term = 0; term < 3; ++term) {
                const uint2 b = wimg[((s * NT + nt) * 3 + term) * kWarp + lane];
#pragma unroll
                for (int mt = 0; mt < kRmMT; ++mt) mma16816<T>(acc[mt][nt], a[mt], b.x, b.y);
              }
          }
        }
      }
    }
    // epilogue: row (mt, hh) holds columns nt*8 + 2qp + {0,1} in acc[mt][nt][2hh + {0,1}]
#pragma unroll
    for (int mt = 0; mt < kRmMT; ++mt)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float ss = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          acc[mt][nt][2 * hh] *= inv_g;
          acc[mt][nt][2 * hh + 1] *= inv_g;
          ss += acc[mt][nt][2 * hh] * acc[mt][nt][2 * hh] + acc[mt][nt][2 * hh + 1] * acc[mt][nt][2 * hh + 1];
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        const float nrm = fmaxf(sqrtf(ss), 1e-12f);
        if (ok[mt][hh]) {
          const int64_t row = task * (16 * kRmMT) + 16 * mt + 8 * hh + gq;
          float* out = p.out + row * (NT * 8) + 2 * qp;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            *reinterpret_cast<float2*>(out + nt * 8) =
                make_float2(acc[mt][nt][2 * hh] / nrm, acc[mt][nt][2 * hh + 1] / nrm);
        }
      }
  }
}

// Codebook rows -> L2-normalised fp32 copy [heads][n_codes][d_s].
template <typename TW>
__global__ void codebook_normalize_kernel(const TW* cb, float* out, int64_t rows, int d_s) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarp) + warp;
  if (row >= rows) return;
  const float v0 = lane < d_s ? Elem<TW>::to_f(cb[row * d_s + lane]) : 0.f;
  const float v1 = lane + kWarp < d_s ? Elem<TW>::to_f(cb[row * d_s + lane + kWarp]) : 0.f;
  float ss = v0 * v0 + v1 * v1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float nrm = fmaxf(sqrtf(ss), 1e-12f);
  if (lane < d_s) out[row * d_s + lane] = v0 / nrm;
  if (lane + kWarp < d_s) out[row * d_s + lane + kWarp] = v1 / nrm;
}

// ---------------------------------------------------------------------------
// K1 (CUDA-core version): one thread per route row, scanning every code of its
// head in increasing code order with a register top-K list.  The codebook
// streams through shared memory in chunks; every thread of the block reads
// the same code at the same time (broadcast).
// ---------------------------------------------------------------------------
constexpr int kSelThreads = 128;
constexpr int kSelChunk = 128;   // codes per shared-memory chunk

template <int KMAX, int DS>
__global__ void __launch_bounds__(kSelThreads) code_select_kernel(CodeSelectParams p) {
  __shared__ __align__(16) float cbs[kSelChunk * DS];
  const int64_t tiles_per_head = cdiv(p.n_rows, kSelThreads);
  const int64_t bh = blockIdx.x / tiles_per_head;        // bat * h_kv + h
  const int64_t tile = blockIdx.x % tiles_per_head;
  const int h = static_cast<int>(bh % p.h_kv);
  const int64_t bat = bh / p.h_kv;
  const int64_t i = tile * kSelThreads + threadIdx.x;
  const bool active = i < p.n_rows;
  const int64_t row = bh * p.n_rows + (active ? i : 0);
  float r[DS];
#pragma unroll
  for (int e = 0; e < DS; e += 4) {
    const float4 v = *reinterpret_cast<const float4*>(p.route + row * DS + e);
    r[e] = v.x; r[e + 1] = v.y; r[e + 2] = v.z; r[e + 3] = v.w;
  }
  TopList<KMAX> top;
  top.init();
  const float* cb = p.codebook + static_cast<int64_t>(p.codebook_heads == 1 ? 0 : h) *
                                     p.n_codes * DS;
  const bool unit_temp = p.temperature == 1.0f;
  for (int c0 = 0; c0 < p.n_codes; c0 += kSelChunk) {
    const int cn = min(kSelChunk, p.n_codes - c0);
    __syncthreads();
    for (int t = threadIdx.x * 4; t < cn * DS; t += kSelThreads * 4)
      *reinterpret_cast<float4*>(cbs + t) =
          *reinterpret_cast<const float4*>(cb + static_cast<int64_t>(c0) * DS + t);
    __syncthreads();
    for (int c = 0; c < cn; ++c) {
      const float4* cv = reinterpret_cast<const float4*>(cbs + c * DS);
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < DS / 4; ++e) {
        const float4 w = cv[e];
        s = fmaf(r[4 * e], w.x, s);
        s = fmaf(r[4 * e + 1], w.y, s);
        s = fmaf(r[4 * e + 2], w.z, s);
        s = fmaf(r[4 * e + 3], w.w, s);
      }
      if (!unit_temp) s = s / p.temperature;
      top.push(s, static_cast<uint32_t>(c0 + c));
    }
  }
  if (!active) return;
  // codes out: [bat][i][h][kk]
  int32_t* out = p.codes + ((bat * p.n_rows + i) * p.h_kv + h) * p.kk;
#pragma unroll
  for (int t = 0; t < KMAX; ++t)
    if (t < p.kk) out[t] = top.index(t);
}

// Selection on fed scores: the same TopList with the same push order.
template <int KMAX>
__global__ void select_from_scores_kernel(const float* scores, int64_t rows, int n_cols, int kk,
                                          int32_t* out) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  TopList<KMAX> top;
  top.init();
  const float* s = scores + r * n_cols;
  for (int c = 0; c < n_cols; ++c) {
    top.push(s[c], static_cast<uint32_t>(c));
  }
#pragma unroll
  for (int t = 0; t < KMAX; ++t)
    if (t < kk) out[r * kk + t] = top.index(t);
}

// ---------------------------------------------------------------------------
// host-side launchers
// ---------------------------------------------------------------------------
template <typename T, typename TW, int NT>
static cudaError_t launch_route_project_mma_t(const RouteProjectParams& p, int sms, cudaStream_t st) {
  auto kern = p.rope_cos ? route_project_mma_kernel<T, TW, NT, true> : route_project_mma_kernel<T, TW, NT, false>;
  const size_t smem = static_cast<size_t>(p.d / 16) * NT * 3 * kWarp * sizeof(uint2);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 1;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kRmWarps * kWarp, smem);
  if (e != cudaSuccess) return e;
  const int64_t tasks = cdiv(p.rows, 16 * kRmMT);
  int64_t blocks = cdiv(tasks, kRmWarps);
  const int64_t cap = static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1);
  if (blocks > cap) blocks = cap;
  kern<<<static_cast<unsigned>(blocks), kRmWarps * kWarp, smem, st>>>(p);
  return cudaGetLastError();
}

template <typename T, typename TW>
static cudaError_t launch_route_project_mma_w(const RouteProjectParams& p, int sms, cudaStream_t st) {
  switch (p.d_s) {
    case 8: return launch_route_project_mma_t<T, TW, 1>(p, sms, st);
    case 16: return launch_route_project_mma_t<T, TW, 2>(p, sms, st);
    case 32: return launch_route_project_mma_t<T, TW, 4>(p, sms, st);
    default: return launch_route_project_mma_t<T, TW, 8>(p, sms, st);
  }
}

// The tensor-core projection takes 16-bit inputs with d a multiple of 32 and
// d_s in {8, 16, 32, 64}; everything else runs the FMA version.
static bool route_project_mma_ok(const RouteProjectParams& p, ssa_dtype xt) {
  return (xt == SSA_BF16 || xt == SSA_F16) && p.d % 32 == 0 && p.d >= 32 &&
         (p.d_s == 8 || p.d_s == 16 || p.d_s == 32 || p.d_s == 64);
}

// RoPE on load: the tensor-core projection with all of a row's chunks in one
// pass (d = 64 or 128).
bool route_project_rope_supported(int d, int d_s, ssa_dtype xt) {
  return (xt == SSA_BF16 || xt == SSA_F16) && (d == 64 || d == 128) &&
         (d_s == 8 || d_s == 16 || d_s == 32 || d_s == 64);
}

cudaError_t launch_route_project(const RouteProjectParams& p, ssa_dtype xt, ssa_dtype wt,
                                 cudaStream_t st) {
  if (p.rows == 0) return cudaSuccess;
  if (p.rope_cos && !route_project_rope_supported(p.d, p.d_s, xt)) return cudaErrorInvalidValue;
  if (route_project_tc_supported(p, xt, wt)) return launch_route_project_tc(p, xt, wt, st);
  if (route_project_mma_ok(p, xt)) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (xt == SSA_BF16 && wt == SSA_BF16) return launch_route_project_mma_w<__nv_bfloat16, __nv_bfloat16>(p, sms, st);
    if (xt == SSA_BF16 && wt == SSA_F32) return launch_route_project_mma_w<__nv_bfloat16, float>(p, sms, st);
    if (xt == SSA_F16 && wt == SSA_F16) return launch_route_project_mma_w<__half, __half>(p, sms, st);
    if (xt == SSA_F16 && wt == SSA_F32) return launch_route_project_mma_w<__half, float>(p, sms, st);
  }
  const int threads = kRpThreads;
  const size_t smem = (static_cast<size_t>(p.d) * p.d_s + static_cast<size_t>(kRpRows) * p.d) * sizeof(float);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t blocks = cdiv(p.rows, kRpRows);
  blocks = blocks > static_cast<int64_t>(sms) * 4 ? static_cast<int64_t>(sms) * 4 : blocks;
  if (blocks < 1) return cudaSuccess;
#define SSA_RP(T, TW)                                                                       \
  do {                                                                                      \
    auto kern = p.d_s > kWarp ? route_project_kernel<T, TW, true> : route_project_kernel<T, TW, false>; \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);     \
    kern<<<(unsigned)blocks, threads, smem, st>>>(p);                                       \
  } while (0)
  if (xt == SSA_F32 && wt == SSA_F32) SSA_RP(float, float);
  else if (xt == SSA_BF16 && wt == SSA_BF16) SSA_RP(__nv_bfloat16, __nv_bfloat16);
  else if (xt == SSA_BF16 && wt == SSA_F32) SSA_RP(__nv_bfloat16, float);
  else if (xt == SSA_F16 && wt == SSA_F16) SSA_RP(__half, __half);
  else if (xt == SSA_F16 && wt == SSA_F32) SSA_RP(__half, float);
  else if (xt == SSA_F32 && wt == SSA_BF16) SSA_RP(float, __nv_bfloat16);
  else return cudaErrorInvalidValue;
#undef SSA_RP
  return cudaGetLastError();
}

cudaError_t launch_codebook_normalize(const void* cb, ssa_dtype wt, float* out, int64_t rows,
                                      int d_s, cudaStream_t st) {
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>(cdiv(rows, threads / kWarp));
  if (blocks == 0) return cudaSuccess;
  if (wt == SSA_F32)
    codebook_normalize_kernel<float><<<blocks, threads, 0, st>>>(static_cast<const float*>(cb), out, rows, d_s);
  else if (wt == SSA_BF16)
    codebook_normalize_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(cb), out, rows, d_s);
  else
    codebook_normalize_kernel<__half><<<blocks, threads, 0, st>>>(static_cast<const __half*>(cb), out, rows, d_s);
  return cudaGetLastError();
}

template <int DS>
static cudaError_t launch_code_select_ds(const CodeSelectParams& p, cudaStream_t st) {
  const int64_t blocks = p.batch_heads * cdiv(p.n_rows, kSelThreads);
  if (blocks == 0) return cudaSuccess;
  if (p.kk <= 4) code_select_kernel<4, DS><<<(unsigned)blocks, kSelThreads, 0, st>>>(p);
  else if (p.kk <= 8) code_select_kernel<8, DS><<<(unsigned)blocks, kSelThreads, 0, st>>>(p);
  else if (p.kk <= 16) code_select_kernel<16, DS><<<(unsigned)blocks, kSelThreads, 0, st>>>(p);
  else code_select_kernel<32, DS><<<(unsigned)blocks, kSelThreads, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_code_select(const CodeSelectParams& p, cudaStream_t st) {
  switch (p.d_s) {
    case 4: return launch_code_select_ds<4>(p, st);
    case 8: return launch_code_select_ds<8>(p, st);
    case 16: return launch_code_select_ds<16>(p, st);
    case 32: return launch_code_select_ds<32>(p, st);
    case 64: return launch_code_select_ds<64>(p, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_select_from_scores(const float* scores, int64_t rows, int n_cols, int kk,
                                      int32_t* out, cudaStream_t st) {
  const int threads = 128;
  const unsigned blocks = static_cast<unsigned>(cdiv(rows, threads));
  if (blocks == 0) return cudaSuccess;
  if (kk <= 4) select_from_scores_kernel<4><<<blocks, threads, 0, st>>>(scores, rows, n_cols, kk, out);
  else if (kk <= 8) select_from_scores_kernel<8><<<blocks, threads, 0, st>>>(scores, rows, n_cols, kk, out);
  else if (kk <= 16) select_from_scores_kernel<16><<<blocks, threads, 0, st>>>(scores, rows, n_cols, kk, out);
  else select_from_scores_kernel<32><<<blocks, threads, 0, st>>>(scores, rows, n_cols, kk, out);
  return cudaGetLastError();
}

}  // namespace ssa
