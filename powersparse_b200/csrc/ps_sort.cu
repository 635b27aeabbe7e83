// Hand-written device scan and stable LSD radix sort (sm_100a).
//
// Radix pass layout: a tile is 4096 consecutive elements (256 threads x 16).
//   1. radix_tile_hist   : per-tile digit counts, stored digit-major
//                          (counts[d * tiles + t]) so that
//   2. exclusive_scan    : over that array yields, for every (digit, tile),
//                          the global output position of its first element;
//   3. radix_scatter     : re-reads the tile, ranks every element among the
//                          equal-digit elements before it (warp strips in order,
//                          lanes in order: __match_any_sync peers), and writes it.
// Which buffer pair holds the data is a device word per pass (`side`), read by the
// kernels of the pass; the scatter writes the next pass's word.  So a sort queues
// all its passes without a host round trip, and a pass whose digit is constant is
// skipped on the device (every block sees the digit totals in the scanned counts).
// Stability: tiles are ordered, warps own consecutive 512-element strips of a
// tile, and within a 32-element chunk the rank counts lower lanes only.
#include "ps_common.cuh"
#include "ps_sort.cuh"

#include <algorithm>
#include <vector>

namespace psb {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T>
__device__ T block_exclusive_scan(T value, T* warp_sums, T& block_total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T inc = value;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    T other = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += other;
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    T w = lane < (kScanThreads / 32) ? warp_sums[lane] : T(0);
    T winc = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      T other = __shfl_up_sync(0xffffffffu, winc, d);
      if (lane >= d) winc += other;
    }
    if (lane < (kScanThreads / 32)) warp_sums[lane] = winc - w;
    if (lane == (kScanThreads / 32) - 1) warp_sums[kScanThreads / 32] = winc;
  }
  __syncthreads();
  const T result = inc - value + warp_sums[warp];
  block_total = warp_sums[kScanThreads / 32];
  __syncthreads();
  return result;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_tile_reduce(const T* __restrict__ in, size_t n,
                                                                 T* __restrict__ partial) {
  __shared__ T warp_sums[kScanThreads / 32 + 1];
  const size_t base = size_t(blockIdx.x) * kScanTile;
  T sum = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const size_t idx = base + size_t(i) * kScanThreads + threadIdx.x;
    if (idx < n) sum += in[idx];
  }
  T total;
  block_exclusive_scan(sum, warp_sums, total);
  if (threadIdx.x == 0) partial[blockIdx.x] = total;
}

template <typename T>
__global__ void __launch_bounds__(kScanThreads) scan_tile_apply(const T* in, T* out, size_t n,
                                                                const T* __restrict__ partial) {
  __shared__ T warp_sums[kScanThreads / 32 + 1];
  const size_t base = size_t(blockIdx.x) * kScanTile + size_t(threadIdx.x) * kScanItems;
  T v[kScanItems];
  T sum = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const size_t idx = base + i;
    v[i] = idx < n ? in[idx] : T(0);
    sum += v[i];
  }
  T total;
  T run = block_exclusive_scan(sum, warp_sums, total) + (partial ? partial[blockIdx.x] : T(0));
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    const size_t idx = base + i;
    if (idx < n) out[idx] = run;
    run += v[i];
  }
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == kScanThreads - 1) out[n] = run;
}

constexpr int kSortThreads = 256;
constexpr int kSortItems = 16;
constexpr int kSortTile = kSortThreads * kSortItems;  // 4096
constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kSortWarps = kSortThreads / 32;
constexpr int kStrip = kSortTile / kSortWarps;  // 512 consecutive elements per warp
static_assert(kSortThreads == kRadix, "one thread per digit in the per-block digit loops");

template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_tile_hist(const K* __restrict__ keys0,
                                                                const K* __restrict__ keys1,
                                                                const int* __restrict__ side, size_t n,
                                                                int shift, uint32_t* __restrict__ counts,
                                                                size_t tiles) {
  const K* __restrict__ keys = *side ? keys1 : keys0;
  __shared__ uint32_t hist[kRadix];
  hist[threadIdx.x] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const size_t base = size_t(blockIdx.x) * kSortTile;
#pragma unroll 4
  for (int i = 0; i < kSortItems; ++i) {
    const size_t idx = base + size_t(i) * kSortThreads + threadIdx.x;
    const uint32_t d = idx < n ? uint32_t(keys[idx] >> shift) & (kRadix - 1) : uint32_t(kRadix);
    const uint32_t peers = __match_any_sync(0xffffffffu, d);
    if (d < kRadix && lane == __ffs(peers) - 1) atomicAdd(&hist[d], uint32_t(__popc(peers)));
  }
  __syncthreads();
  counts[size_t(threadIdx.x) * tiles + blockIdx.x] = hist[threadIdx.x];
}

// offsets: the scanned digit-major tile counts, kRadix * tiles + 1 entries (the last
// is n), so digit d's first output position is offsets[d * tiles].  side[0]: where
// the data is; side[1] (written by block 0): where this pass leaves it.
template <typename K>
__global__ void __launch_bounds__(kSortThreads) radix_scatter(K* keys0, uint32_t* vals0, K* keys1,
                                                              uint32_t* vals1, int* side, size_t n,
                                                              int shift,
                                                              const uint32_t* __restrict__ offsets,
                                                              size_t tiles) {
  __shared__ uint32_t whist[kSortWarps][kRadix];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cur = side[0];
  {
    // kSortThreads == kRadix: thread d looks at digit d's total.
    const int d = threadIdx.x;
    const uint32_t total = offsets[size_t(d + 1) * tiles] - offsets[size_t(d) * tiles];
    const bool constant = __syncthreads_or(size_t(total) == n) != 0;
    if (blockIdx.x == 0 && threadIdx.x == 0) side[1] = constant ? cur : 1 - cur;
    if (constant) return;  // every key has this digit: the pass is the identity
  }
  const K* __restrict__ kin = cur ? keys1 : keys0;
  const uint32_t* __restrict__ vin = cur ? vals1 : vals0;
  K* __restrict__ kout = cur ? keys0 : keys1;
  uint32_t* __restrict__ vout = cur ? vals0 : vals1;
  for (int i = threadIdx.x; i < kSortWarps * kRadix; i += kSortThreads) (&whist[0][0])[i] = 0;
  __syncthreads();
  const size_t base = size_t(blockIdx.x) * kSortTile + size_t(warp) * kStrip;
  K key[kSortItems];
  uint32_t val[kSortItems];
  uint32_t dig[kSortItems];
#pragma unroll
  for (int c = 0; c < kSortItems; ++c) {
    const size_t idx = base + size_t(c) * 32 + lane;
    if (idx < n) {
      key[c] = kin[idx];
      val[c] = vin[idx];
      dig[c] = uint32_t(key[c] >> shift) & (kRadix - 1);
    } else {
      key[c] = 0;
      val[c] = 0;
      dig[c] = kRadix;
    }
  }
#pragma unroll
  for (int c = 0; c < kSortItems; ++c) {
    const uint32_t peers = __match_any_sync(0xffffffffu, dig[c]);
    if (dig[c] < kRadix && lane == __ffs(peers) - 1) whist[warp][dig[c]] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  {
    const int d = threadIdx.x;  // kSortThreads == kRadix
    uint32_t run = offsets[size_t(d) * tiles + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kSortWarps; ++w) {
      const uint32_t t = whist[w][d];
      whist[w][d] = run;
      run += t;
    }
  }
  __syncthreads();
  const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
  for (int c = 0; c < kSortItems; ++c) {
    const uint32_t peers = __match_any_sync(0xffffffffu, dig[c]);
    if (dig[c] < kRadix) {
      const uint32_t pos = whist[warp][dig[c]] + __popc(peers & lt_mask);
      kout[pos] = key[c];
      vout[pos] = val[c];
    }
    __syncwarp();
    if (dig[c] < kRadix && lane == __ffs(peers) - 1) whist[warp][dig[c]] += __popc(peers);
    __syncwarp();
  }
}

__global__ void take_from_alt_kernel(const int* __restrict__ side, const uint32_t* __restrict__ alt,
                                     uint32_t* __restrict__ primary, size_t n) {
  if (!*side) return;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    primary[i] = alt[i];
}

__global__ void iota_kernel(uint32_t* v, size_t n) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    v[i] = uint32_t(i);
}

}  // namespace

template <typename T>
void exclusive_scan(const T* in, T* out, size_t n, cudaStream_t stream) {
  if (n == 0) {
    PSB_CUDA(cudaMemsetAsync(out, 0, sizeof(T), stream));
    return;
  }
  const size_t tiles = (n + kScanTile - 1) / kScanTile;
  if (tiles == 1) {
    scan_tile_apply<T><<<1, kScanThreads, 0, stream>>>(in, out, n, nullptr);
    PSB_LAUNCH_CHECK();
    return;
  }
  StreamArray<T> partial(tiles + 1, stream);
  scan_tile_reduce<T><<<unsigned(tiles), kScanThreads, 0, stream>>>(in, n, partial.get());
  PSB_LAUNCH_CHECK();
  exclusive_scan<T>(partial.get(), partial.get(), tiles, stream);
  scan_tile_apply<T><<<unsigned(tiles), kScanThreads, 0, stream>>>(in, out, n, partial.get());
  PSB_LAUNCH_CHECK();
}

int radix_passes(size_t n, int begin_bit, int end_bit) {
  if (n <= 1 || end_bit <= begin_bit) return 0;
  return (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
}

template <typename K>
void radix_sort_pairs_async(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt, size_t n,
                            int begin_bit, int end_bit, int* side, cudaStream_t stream) {
  const int passes = radix_passes(n, begin_bit, end_bit);
  if (passes == 0) return;
  if (n >= (size_t(1) << 32)) throw std::invalid_argument("radix sort: more than 2^32 - 1 elements");
  const size_t tiles = (n + kSortTile - 1) / kSortTile;
  StreamArray<uint32_t> offsets(size_t(kRadix) * tiles + 1, stream);
  for (int p = 0; p < passes; ++p) {
    const int shift = begin_bit + p * kRadixBits;
    radix_tile_hist<K><<<unsigned(tiles), kSortThreads, 0, stream>>>(keys, keys_alt, side + p, n, shift,
                                                                      offsets.get(), tiles);
    PSB_LAUNCH_CHECK();
    exclusive_scan<uint32_t>(offsets.get(), offsets.get(), size_t(kRadix) * tiles, stream);
    radix_scatter<K><<<unsigned(tiles), kSortThreads, 0, stream>>>(keys, vals, keys_alt, vals_alt, side + p, n,
                                                                    shift, offsets.get(), tiles);
    PSB_LAUNCH_CHECK();
  }
}

template <typename K>
bool radix_sort_pairs(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt, size_t n,
                      int begin_bit, int end_bit, cudaStream_t stream) {
  const int passes = radix_passes(n, begin_bit, end_bit);
  if (passes == 0) return false;
  StreamArray<int> side(size_t(passes) + 1, stream);
  PSB_CUDA(cudaMemsetAsync(side.get(), 0, sizeof(int), stream));
  radix_sort_pairs_async<K>(keys, vals, keys_alt, vals_alt, n, begin_bit, end_bit, side.get(), stream);
  int h_side = 0;
  PSB_CUDA(cudaMemcpyAsync(&h_side, side.get() + passes, sizeof(int), cudaMemcpyDeviceToHost, stream));
  PSB_CUDA(cudaStreamSynchronize(stream));
  return h_side != 0;
}

void take_from_alt(const int* side, const uint32_t* alt, uint32_t* primary, size_t n, cudaStream_t stream) {
  if (!n) return;
  const unsigned blocks = unsigned(std::min<size_t>((n + 255) / 256, size_t(8) * device_sms()));
  take_from_alt_kernel<<<blocks, 256, 0, stream>>>(side, alt, primary, n);
  PSB_LAUNCH_CHECK();
}

void iota_u32(uint32_t* vals, size_t n, cudaStream_t stream) {
  if (!n) return;
  const unsigned blocks = unsigned(std::min<size_t>((n + 255) / 256, size_t(32) * device_sms()));
  iota_kernel<<<blocks, 256, 0, stream>>>(vals, n);
  PSB_LAUNCH_CHECK();
}

template void exclusive_scan<int32_t>(const int32_t*, int32_t*, size_t, cudaStream_t);
template void exclusive_scan<uint32_t>(const uint32_t*, uint32_t*, size_t, cudaStream_t);
template void exclusive_scan<int64_t>(const int64_t*, int64_t*, size_t, cudaStream_t);
template void radix_sort_pairs_async<uint32_t>(uint32_t*, uint32_t*, uint32_t*, uint32_t*, size_t, int, int,
                                               int*, cudaStream_t);
template void radix_sort_pairs_async<uint64_t>(uint64_t*, uint32_t*, uint64_t*, uint32_t*, size_t, int, int,
                                               int*, cudaStream_t);
template bool radix_sort_pairs<uint32_t>(uint32_t*, uint32_t*, uint32_t*, uint32_t*, size_t, int, int,
                                         cudaStream_t);
template bool radix_sort_pairs<uint64_t>(uint64_t*, uint32_t*, uint64_t*, uint32_t*, size_t, int, int,
                                         cudaStream_t);

}  // namespace psb
