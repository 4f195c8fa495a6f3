// K0 on the 5th-generation tensor cores: the routing projection of 16-bit
// queries and keys, fed by TMA.
//
// Reference: ssa/router.py:102-118 -- q_route = mean_g W_qr q_g (the g query
// heads of a KV group), k_route = W_kr k, then F.normalize.  The group mean is
// one linear map, so a KV group's route is one GEMM row with K = g*d: the
// group's g heads lie side by side in a row of q ([B, n, h_q, d] with the
// heads contiguous), and B repeats W along K.  The 1/g factor is dropped: it
// does not change the normalised vector.
//
// Exact products: W (fp32) is split into three terms of the input type,
// w = w0 + w1 + w2 (exact for bf16), and B holds them side by side on the N
// axis, N = 3 * d_s.  Every product x * w_t is exact in the fp32 accumulator;
// the epilogue adds the three partial sums of a route component and
// normalises.
//
// Per CTA (persistent, one per SM, tiles of 128 rows of one (bat, h) taken
// round-robin):
//   warp 0     TMA producer: 3-D tensor copies of 128 rows x 64 elements
//              (128-byte rows, SWIZZLE_128B) into a 6-stage shared-memory ring;
//   warp 1     TMEM allocation and the single-thread tcgen05.mma issuer,
//              M = 128, N = 3 * d_s, K = 16, into two TMEM accumulators;
//   warps 2-5  epilogue: one row per thread (its TMEM lane), three groups of
//              d_s columns summed, L2-normalised, stored as d_s fp32.
// B (the W terms, K-major SWIZZLE_NONE, d columns) is built once per CTA in
// shared memory; chunk c of a row uses W columns (64 c) mod d.
//
// Every wait is bounded (about one second); on expiry the CTA records
// SSA_DEVICE_TIMEOUT, stops issuing, waits (bounded) for its copies and MMAs
// in flight, frees TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"
#include "tc_utils.cuh"

namespace ssa {
namespace rtc {

using namespace tc;

constexpr int kM = 128;            // rows per tile (TMEM lanes)
constexpr int kKC = 64;            // K elements per TMA box and pipeline stage (128 bytes)
constexpr int kStages = 6;
constexpr int kStageBytes = kM * kKC * 2;
constexpr int kEpiWarps = 4;
constexpr int kThreads = 64 + 32 * kEpiWarps;

template <int DS>
struct RtGeo {
  static constexpr int N = 3 * DS;                            // w0 | w1 | w2
  static constexpr int TCOLS = N <= 64 ? 64 : (N <= 128 ? 128 : 256);   // TMEM columns per buffer
  static constexpr int B_LBO = (N / 8) * 128;                 // bytes between 16-byte K groups of B
};

struct RouteTcParams {
  float* out;                       // [batch_heads * n_rows, d_s]
  const void* w;                    // [d_s, d] (TW)
  int32_t* status;
  int64_t n_rows, tiles_per_head, total_tiles;
  int h_kv, group, d;
};

__device__ __forceinline__ uint32_t b_off(int n, int k, int lbo) {
  return static_cast<uint32_t>((k >> 3) * lbo + (n >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2);
}

template <typename T, typename TW, int DS>
__global__ void __launch_bounds__(kThreads, 1) route_project_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                       RouteTcParams p) {
  using G = RtGeo<DS>;
  constexpr uint32_t kIdesc = idesc_f16(kM, G::N, std::is_same<T, __nv_bfloat16>::value);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* a_ring = base;                                   // kStages x 16 KB, 1024-aligned
  unsigned char* b_img = a_ring + kStages * kStageBytes;          // N x d x 2 bytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(b_img + G::N * p.d * 2);
  const uint32_t full = smem_u32(bars);
  const uint32_t empty = full + 8 * kStages;
  const uint32_t tfull = empty + 8 * kStages;
  const uint32_t tempty = tfull + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int kc_per_tile = p.group * p.d / kKC;

  // ---- B: the three terms of W, K-major, SWIZZLE_NONE ----
  for (int idx = threadIdx.x; idx < G::N * p.d; idx += blockDim.x) {
    const int n = idx / p.d, k = idx % p.d;
    const int t = n / DS, c = n % DS;
    const float w = Elem<TW>::to_f(static_cast<const TW*>(p.w)[c * p.d + k]);
    const T w0 = Elem<T>::from_f(w);
    const float r1 = w - Elem<T>::to_f(w0);
    const T w1 = Elem<T>::from_f(r1);
    const T w2 = Elem<T>::from_f(r1 - Elem<T>::to_f(w1));
    *reinterpret_cast<T*>(b_img + b_off(n, k, G::B_LBO)) = t == 0 ? w0 : (t == 1 ? w1 : w2);
  }
  fence_proxy_async();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + 8 * s, 1);
      mbar_init(empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + 8 * b, 1);
      mbar_init(tempty + 8 * b, kEpiWarps);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_tensormap(&xmap);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(2 * G::TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem_base = *tmem_slot;
  auto fail = [&]() {
    *abort_flag = 1;
    if (p.status) atomicOr(p.status, SSA_DEVICE_TIMEOUT);
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int64_t g = 0;
      bool stop = false;
      for (int64_t tile = blockIdx.x; tile < p.total_tiles && !stop; tile += gridDim.x) {
        const int64_t bh = tile / p.tiles_per_head;
        const int i0 = static_cast<int>((tile % p.tiles_per_head) * kM);
        const int bat = static_cast<int>(bh / p.h_kv), h = static_cast<int>(bh % p.h_kv);
        const int x0 = h * p.group * p.d;
        for (int kc = 0; kc < kc_per_tile; ++kc, ++g) {
          const int s = static_cast<int>(g % kStages);
          const uint32_t ph = static_cast<uint32_t>((g / kStages) & 1);
          if (*abort_flag || !mbar_wait(empty + 8 * s, ph ^ 1u)) { fail(); stop = true; break; }
          mbar_expect_tx(full + 8 * s, kStageBytes);
          tma_load_3d(smem_u32(a_ring + s * kStageBytes), &xmap, x0 + kc * kKC, i0, bat, full + 8 * s);
        }
      }
      // every issued copy lands before the CTA exits
      for (int64_t r = g - 1; r >= 0 && r >= g - kStages; --r)
        mbar_wait(full + 8 * static_cast<int>(r % kStages), static_cast<uint32_t>((r / kStages) & 1));
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int64_t g = 0, tl = 0;
      bool issued = false;
      const uint32_t b_base = smem_u32(b_img);
      for (int64_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++tl) {
        const int buf = static_cast<int>(tl & 1);
        if (*abort_flag || !mbar_wait(tempty + 8 * buf, static_cast<uint32_t>(((tl >> 1) & 1) ^ 1u))) {
          fail();
          break;
        }
        fence_after();
        const uint32_t d_tmem = tmem_base + buf * G::TCOLS;
        bool stop = false;
        for (int kc = 0; kc < kc_per_tile; ++kc, ++g) {
          const int s = static_cast<int>(g % kStages);
          if (*abort_flag || !mbar_wait(full + 8 * s, static_cast<uint32_t>((g / kStages) & 1))) {
            fail();
            stop = true;
            break;
          }
          fence_after();
          const uint32_t a_base = smem_u32(a_ring + s * kStageBytes);
          const int kw = (kc * kKC) % p.d;                  // W column of the chunk's first element
#pragma unroll
          for (int ks = 0; ks < kKC / 16; ++ks) {
            const uint64_t ad = sdesc(a_base + ks * 32, 0, 1024, 2);          // SWIZZLE_128B, K-major
            const uint64_t bd = sdesc(b_base + ((kw + ks * 16) >> 3) * G::B_LBO, G::B_LBO, 128, 0);
            mma_f16(d_tmem, ad, bd, kIdesc, (kc > 0 || ks > 0) ? 1u : 0u);
          }
          mma_commit(empty + 8 * s);                          // the stage is free once these MMAs ran
          issued = true;
        }
        if (stop) break;
        mma_commit(tfull + 8 * buf);
      }
      // drain: the last commit arrives only after every MMA issued before it
      if (issued) {
        const int64_t r = g - 1;
        mbar_wait(empty + 8 * static_cast<int>(r % kStages), static_cast<uint32_t>((r / kStages) & 1));
      }
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;                           // TMEM lanes 32 * quarter .. + 31
    const int r = quarter * 32 + lane;
    int64_t tl = 0;
    for (int64_t tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++tl) {
      const int buf = static_cast<int>(tl & 1);
      if (*abort_flag || !mbar_wait(tfull + 8 * buf, static_cast<uint32_t>((tl >> 1) & 1))) {
        fail();
        break;
      }
      fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * G::TCOLS;
      float s[DS];
      if constexpr (DS == 16) {
        uint32_t v[3][16];
        tmem_ld16_async(taddr, v[0]);
        tmem_ld16_async(taddr + 16, v[1]);
        tmem_ld16_async(taddr + 32, v[2]);
        tmem_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j)
          s[j] = (__uint_as_float(v[0][j]) + __uint_as_float(v[1][j])) + __uint_as_float(v[2][j]);
      } else {
#pragma unroll
        for (int c0 = 0; c0 < DS; c0 += 32) {
          uint32_t v[3][32];
          tmem_ld32_async(taddr + c0, v[0]);
          tmem_ld32_async(taddr + DS + c0, v[1]);
          tmem_ld32_async(taddr + 2 * DS + c0, v[2]);
          tmem_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            s[c0 + j] = (__uint_as_float(v[0][j]) + __uint_as_float(v[1][j])) + __uint_as_float(v[2][j]);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty + 8 * buf);          // the accumulator may be overwritten
      const int64_t bh = tile / p.tiles_per_head;
      const int64_t i = (tile % p.tiles_per_head) * kM + r;
      if (i < p.n_rows) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DS; ++j) ss = fmaf(s[j], s[j], ss);
        const float nrm = fmaxf(sqrtf(ss), 1e-12f);          // F.normalize: x / max(||x||, eps)
        float4* dst = reinterpret_cast<float4*>(p.out + (bh * p.n_rows + i) * DS);
#pragma unroll
        for (int j = 0; j < DS; j += 4)
          dst[j / 4] = make_float4(s[j] / nrm, s[j + 1] / nrm, s[j + 2] / nrm, s[j + 3] / nrm);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(2 * G::TCOLS));
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

template <int DS>
size_t smem_bytes(int d) {
  return 1024 + static_cast<size_t>(kStages) * kStageBytes + static_cast<size_t>(RtGeo<DS>::N) * d * 2 + 128;
}

template <typename T, typename TW, int DS>
cudaError_t launch_t(const RouteProjectParams& rp, cudaStream_t st) {
  // rows of x: [B, n_rows, width] with width = h_kv * group * d elements of one row
  const int64_t width = static_cast<int64_t>(rp.h_kv) * rp.group * rp.d;
  const int64_t batch = rp.rows / (static_cast<int64_t>(rp.h_kv) * rp.n_rows);
  CUtensorMap map;
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rp.n_rows),
                              static_cast<cuuint64_t>(batch)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(rp.stride_n) * 2, static_cast<cuuint64_t>(rp.stride_b) * 2};
  const cuuint32_t box[3] = {kKC, kM, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (enc(&map, dt, 3, const_cast<void*>(rp.x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  RouteTcParams p{};
  p.out = rp.out;
  p.w = rp.w;
  p.status = rp.status;
  p.n_rows = rp.n_rows;
  p.tiles_per_head = cdiv(rp.n_rows, kM);
  p.total_tiles = (rp.rows / rp.n_rows) * p.tiles_per_head;
  p.h_kv = rp.h_kv;
  p.group = rp.group;
  p.d = rp.d;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = p.total_tiles < sms ? p.total_tiles : sms;
  const size_t smem = smem_bytes<DS>(rp.d);
  auto kern = route_project_tc_kernel<T, TW, DS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  kern<<<static_cast<unsigned>(grid), kThreads, smem, st>>>(map, p);
  return cudaGetLastError();
}

template <typename T, typename TW>
cudaError_t launch_ds(const RouteProjectParams& rp, cudaStream_t st) {
  switch (rp.d_s) {
    case 16: return launch_t<T, TW, 16>(rp, st);
    case 32: return launch_t<T, TW, 32>(rp, st);
    default: return launch_t<T, TW, 64>(rp, st);
  }
}

}  // namespace rtc

bool route_project_tc_supported(const RouteProjectParams& p, ssa_dtype xt, ssa_dtype wt) {
  if (xt != SSA_BF16 && xt != SSA_F16) return false;
  if (!(wt == SSA_F32 || wt == xt)) return false;
  if (p.rope_cos) return false;                                   // RoPE on load: the mma.sync kernel
  if (!(p.d_s == 16 || p.d_s == 32 || p.d_s == 64)) return false;
  if (p.d % rtc::kKC != 0 || p.d > 256) return false;
  // the group's heads side by side in a row, 16-byte aligned rows
  if (p.stride_h != p.d) return false;
  if ((reinterpret_cast<uintptr_t>(p.x) & 15u) != 0 || (p.stride_n * 2) % 16 != 0 || (p.stride_b * 2) % 16 != 0)
    return false;
  if (p.stride_n < static_cast<int64_t>(p.h_kv) * p.group * p.d) return false;
  if (p.n_rows < 1 || p.rows % (static_cast<int64_t>(p.h_kv) * p.n_rows) != 0) return false;
  return rtc::encode_fn() != nullptr;
}

cudaError_t launch_route_project_tc(const RouteProjectParams& p, ssa_dtype xt, ssa_dtype wt, cudaStream_t st) {
  if (xt == SSA_BF16) {
    return wt == SSA_F32 ? rtc::launch_ds<__nv_bfloat16, float>(p, st)
                         : rtc::launch_ds<__nv_bfloat16, __nv_bfloat16>(p, st);
  }
  return wt == SSA_F32 ? rtc::launch_ds<__half, float>(p, st) : rtc::launch_ds<__half, __half>(p, st);
}

}  // namespace ssa
