// Measurement hook: the L2 read bandwidth this GPU sustains on a buffer that
// fits in L2 -- the denominator the benchmark uses for the gather-bound
// kernels, whose K / V rows are served from L2.  No reference counterpart.
//
// Each thread streams 16-byte L2-only loads (ld.global.cg: no L1 allocation)
// over the buffer `reps` times, four loads in flight per thread, and folds
// the words into a value that is written only if it matches an impossible
// pattern, so the loads cannot be removed.
#include "common.cuh"
#include "kernels.cuh"

namespace ssa {
namespace {

__global__ void __launch_bounds__(256) l2_read_probe_kernel(const uint4* buf, int64_t n16, int reps,
                                                            unsigned long long* sink) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t acc = 0;
  for (int r = 0; r < reps; ++r) {
    int64_t i = t0;
    for (; i + 3 * stride < n16; i += 4 * stride) {
      const uint4 a = __ldcg(buf + i), b = __ldcg(buf + i + stride), c = __ldcg(buf + i + 2 * stride),
                  d = __ldcg(buf + i + 3 * stride);
      acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n16; i += stride) {
      const uint4 a = __ldcg(buf + i);
      acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
  }
  if (acc == 0x9e3779b9u) atomicAdd(sink, 1ull);
}

}  // namespace

cudaError_t launch_l2_read_probe(const void* buf, size_t bytes, int reps, unsigned long long* sink, cudaStream_t st) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  l2_read_probe_kernel<<<static_cast<unsigned>(sms * 8), 256, 0, st>>>(static_cast<const uint4*>(buf),
                                                                        static_cast<int64_t>(bytes / 16), reps, sink);
  return cudaGetLastError();
}

}  // namespace ssa
