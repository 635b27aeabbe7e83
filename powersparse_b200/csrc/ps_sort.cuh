// Device-wide scan and stable LSD radix sort used by the GPU preprocessing.
//
// The reference sorts with thrust/CUB merge sorts (utils/matrix_utils.cu:522-524,
// 590-592, 609, 616).  Every one of those sorts is a *stable* ordering by an
// integer key, so here they become LSD radix sorts over exactly the key bits in
// use: the same order, in fewer passes over HBM.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace psb {

// out[i] = sum(in[0..i)) for i <= n (so out has n + 1 entries and out[n] is the total).
// in == out is allowed.  T is int32_t, uint32_t or int64_t.
template <typename T>
void exclusive_scan(const T* in, T* out, size_t n, cudaStream_t stream);

// Digit passes that radix_sort_pairs_async makes over n keys for key bits
// [begin_bit, end_bit) (0 when there is nothing to sort).
int radix_passes(size_t n, int begin_bit, int end_bit);

// Stable sort of (keys, vals) by key bits [begin_bit, end_bit), queued on `stream`
// without waiting for the device.  The data moves between the pairs (keys, vals)
// and (keys_alt, vals_alt), and which pair holds it lives in device memory: side[0]
// (0 = the first pair, 1 = the alternates) says where the data is before the sort,
// and digit pass p writes side[p + 1].  A pass in which every key has the same digit
// leaves the data where it is.  After the sort, side[radix_passes(n, begin_bit,
// end_bit)] says where the sorted data is.  K is uint32_t or uint64_t.
template <typename K>
void radix_sort_pairs_async(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt, size_t n,
                            int begin_bit, int end_bit, int* side, cudaStream_t stream);

// radix_sort_pairs_async on data that starts in (keys, vals); waits for the device
// and returns where the sorted data is (true = the alternates).
template <typename K>
bool radix_sort_pairs(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt, size_t n,
                      int begin_bit, int end_bit, cudaStream_t stream);

// primary[i] = alt[i] for i < n when *side is 1 (the data is in the alternates);
// nothing otherwise.  Queued on `stream` without waiting.
void take_from_alt(const int* side, const uint32_t* alt, uint32_t* primary, size_t n, cudaStream_t stream);

// vals[i] = i.
void iota_u32(uint32_t* vals, size_t n, cudaStream_t stream);

}  // namespace psb
