// The code->key index of a growing key cache (incremental decode).
//
// The reference has no decode path; its design notes say the index is kept
// incrementally so that a decode step does not rescan the whole cache
// (ssa_design.md, "incremental decode").  Layout per (bat, h): bucket c owns
// the slots [start[c], start[c+1]) of `keys` (and of `codes`, each entry's
// four key codes when b == 4) and holds its keys, ascending, in
// [start[c], end[c]).  A rebuild gives every bucket max(slack, size) free
// slots; appending a key writes its b entries at the ends of its b buckets
// (keys arrive in position order, so buckets stay sorted).  `min_free` tracks
// the fewest free slots of any bucket, so that the host knows when the next
// append could overflow and rebuilds first.
//
// The re-score kernels read this layout through RescoreParams::bucket_end.
#include <climits>

#include "common.cuh"
#include "kernels.cuh"

namespace ssa {

namespace {

constexpr int kLayoutThreads = 1024;

// Per (bat, h): bucket capacities from the packed index's sizes, their
// exclusive scan (the starts), the ends, and the minimum free room.
__global__ void __launch_bounds__(kLayoutThreads) decode_layout_kernel(DecodeIndexParams p, const int32_t* ptr) {
  const int64_t bh = blockIdx.x;
  const int32_t* pp = ptr + bh * (p.n_codes + 1);
  int32_t* start = p.start + bh * (p.n_codes + 1);
  int32_t* end = p.end + bh * (p.n_codes + 1);
  __shared__ int32_t warp_sum[kLayoutThreads / kWarp];
  __shared__ int64_t carry;
  __shared__ int32_t fmin[kLayoutThreads / kWarp];
  const int lane = threadIdx.x % kWarp, warp = threadIdx.x / kWarp;
  if (threadIdx.x == 0) carry = 0;
  int my_min = INT_MAX;
  __syncthreads();
  for (int c0 = 0; c0 < p.n_codes; c0 += kLayoutThreads) {
    const int c = c0 + threadIdx.x;
    int count = 0, cap = 0;
    if (c < p.n_codes) {
      count = pp[c + 1] - pp[c];
      cap = count + max(p.slack, count);
      my_min = min(my_min, cap - count);
    }
    int incl = cap;
#pragma unroll
    for (int o = 1; o < kWarp; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == kWarp - 1) warp_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sum[lane];
#pragma unroll
      for (int o = 1; o < kWarp; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sum[lane] = w;                               // inclusive over warps
    }
    __syncthreads();
    const int64_t base = carry + (warp > 0 ? warp_sum[warp - 1] : 0) + (incl - cap);
    if (c < p.n_codes) {
      start[c] = static_cast<int32_t>(base);
      end[c] = static_cast<int32_t>(base + count);
    }
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_sum[kLayoutThreads / kWarp - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    start[p.n_codes] = static_cast<int32_t>(carry < INT_MAX ? carry : static_cast<int64_t>(INT_MAX));
    // the host sized entry_capacity for the worst case; a layout past it is a bug
    if (carry > p.entry_capacity) set_status(p.status, SSA_DEVICE_INDEX_FULL);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) my_min = min(my_min, __shfl_xor_sync(0xffffffffu, my_min, o));
  if (lane == 0) fmin[warp] = my_min;
  __syncthreads();
  if (warp == 0) {
    int m = fmin[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = min(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0 && p.min_free) atomicMin(p.min_free, m);
  }
}

// One warp per bucket: copy the packed bucket into its slots (and, when
// b == 4, each entry's key codes beside it).
__global__ void __launch_bounds__(256) decode_spread_kernel(DecodeIndexParams p, const int32_t* ptr,
                                                            const int32_t* keys) {
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x % kWarp;
  const int64_t bh = blockIdx.y;
  const int c = blockIdx.x * (blockDim.x / kWarp) + warp;
  if (c >= p.n_codes) return;
  const int32_t* pp = ptr + bh * (p.n_codes + 1);
  const int32_t* src = keys + bh * static_cast<int64_t>(p.n) * p.b;
  const int lo = pp[c], hi = pp[c + 1];
  const int s = p.start[bh * (p.n_codes + 1) + c];
  if (s + (hi - lo) > p.entry_capacity) return;         // flagged by the layout kernel
  int32_t* dst = p.keys + bh * p.entry_capacity + s;
  int4* cdst = p.codes ? p.codes + bh * p.entry_capacity + s : nullptr;
  const int bat = static_cast<int>(bh / p.h_kv), h = static_cast<int>(bh % p.h_kv);
  for (int e = lane; e < hi - lo; e += kWarp) {
    const int32_t j = src[lo + e];
    dst[e] = j;
    if (cdst)
      cdst[e] = *reinterpret_cast<const int4*>(p.k_codes + bat * p.k_codes_sb + (static_cast<int64_t>(j) * p.h_kv + h) * 4);
  }
}

// One warp per (bat, h): keys first .. first+count-1 in order, lane m placing
// the entry of the key's code m at the end of that bucket.
__global__ void __launch_bounds__(kWarp) decode_append_kernel(DecodeIndexParams p, int first, int count) {
  const int64_t bh = blockIdx.x;
  const int lane = threadIdx.x;
  const int bat = static_cast<int>(bh / p.h_kv), h = static_cast<int>(bh % p.h_kv);
  const int32_t* start = p.start + bh * (p.n_codes + 1);
  int32_t* end = p.end + bh * (p.n_codes + 1);
  int32_t* keys = p.keys + bh * p.entry_capacity;
  int4* codes = p.codes ? p.codes + bh * p.entry_capacity : nullptr;
  int my_min = INT_MAX;
  for (int t = 0; t < count; ++t) {
    const int j = first + t;
    const int32_t* kc = p.k_codes + bat * p.k_codes_sb + (static_cast<int64_t>(j) * p.h_kv + h) * p.b;
    int c = -1;
    if (lane < p.b) c = checked_code(kc[lane], p.n_codes, p.status);
    // a code repeated within one key is placed once
    bool dup = false;
    for (int m = 0; m < p.b; ++m) {
      const int cm = __shfl_sync(0xffffffffu, c, m);
      dup |= (m < lane) && (cm == c);
    }
    if (lane < p.b && !dup) {
      const int slot = end[c];
      if (slot < start[c + 1]) {
        keys[slot] = j;
        if (codes) codes[slot] = *reinterpret_cast<const int4*>(kc);
        end[c] = slot + 1;
        my_min = min(my_min, start[c + 1] - slot - 1);
      } else {
        set_status(p.status, SSA_DEVICE_INDEX_FULL);
        my_min = 0;
      }
    }
    __syncwarp();                                       // the next key sees these ends
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) my_min = min(my_min, __shfl_xor_sync(0xffffffffu, my_min, o));
  if (lane == 0 && p.min_free && my_min != INT_MAX) atomicMin(p.min_free, my_min);
}

}  // namespace

cudaError_t launch_decode_index_layout(const DecodeIndexParams& p, const int32_t* packed_ptr,
                                       const int32_t* packed_keys, cudaStream_t st) {
  const int64_t bhs = static_cast<int64_t>(p.batch) * p.h_kv;
  decode_layout_kernel<<<static_cast<unsigned>(bhs), kLayoutThreads, 0, st>>>(p, packed_ptr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const dim3 grid(static_cast<unsigned>(cdiv(p.n_codes, 8)), static_cast<unsigned>(bhs));
  decode_spread_kernel<<<grid, 256, 0, st>>>(p, packed_ptr, packed_keys);
  return cudaGetLastError();
}

cudaError_t launch_decode_index_append(const DecodeIndexParams& p, int first, int count, cudaStream_t st) {
  const int64_t bhs = static_cast<int64_t>(p.batch) * p.h_kv;
  decode_append_kernel<<<static_cast<unsigned>(bhs), kWarp, 0, st>>>(p, first, count);
  return cudaGetLastError();
}

}  // namespace ssa
