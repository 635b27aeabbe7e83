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

// Stable sort of (keys, vals) by key bits [begin_bit, end_bit).  Uses the *_alt
// buffers as ping-pong space; on return the sorted data is in (keys, vals) or in
// (keys_alt, vals_alt) as reported by the return value (true = alt).  Digit passes
// in which every key has the same digit are skipped.  K is uint32_t or uint64_t.
template <typename K>
bool radix_sort_pairs(K* keys, uint32_t* vals, K* keys_alt, uint32_t* vals_alt, size_t n,
                      int begin_bit, int end_bit, cudaStream_t stream);

// vals[i] = i.
void iota_u32(uint32_t* vals, size_t n, cudaStream_t stream);

}  // namespace psb
