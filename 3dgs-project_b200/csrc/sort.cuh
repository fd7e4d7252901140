// sort.cuh - device-wide exclusive scan and stable LSD radix sort (internal API).
//
// Both are written for this library instead of calling CUB: the scan feeds the tile-instance and
// bucket offsets, the sort orders the (tile | depth) instance keys. The scan never waits on other
// blocks (reduce-then-scan). The sort is single-sweep per 8-bit digit: its scatter blocks look back
// over counts published by earlier blocks; every such wait is bounded, and a wait that gives up is
// counted on the device and reported by splat_check_device_waits instead of hanging the launch.
#pragma once

#include "common.cuh"

namespace splat {

constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;  // 4096 values per scan block

constexpr int kSortThreads = 256;
#ifndef SPLAT_SORT_ROUNDS
#define SPLAT_SORT_ROUNDS 16
#endif
constexpr int kSortRounds = SPLAT_SORT_ROUNDS;
#ifndef SPLAT_SORT_MIN_BLOCKS
#define SPLAT_SORT_MIN_BLOCKS 3
#endif
constexpr int kSortMinBlocks = SPLAT_SORT_MIN_BLOCKS;  // resident scatter blocks per SM to budget registers for
constexpr int kSortTile = kSortThreads * kSortRounds;  // pairs per sort block
constexpr int kRadixBits = 8;
constexpr int kRadix = 1 << kRadixBits;
constexpr int kMaxPasses = 64 / kRadixBits;

// Workspace needed by scan_exclusive_u32 for n values.
size_t scan_workspace_bytes(long long n);

// out[i] = in[0] + ... + in[i-1]; *total (device pointer, may be null) = sum of all n values.
// in and out may alias.
int scan_exclusive_u32(const uint32_t* in, uint32_t* out, long long n, uint32_t* total, void* ws,
                       size_t ws_bytes, cudaStream_t stream);

// scan_exclusive_u32 with its block sums in a fixed device array instead of a workspace (n at most
// SPLAT_SCAN_NOALLOC_MAX_N); calls on one device share that array.
int scan_exclusive_u32_noalloc(const uint32_t* in, uint32_t* out, long long n, uint32_t* total,
                               cudaStream_t stream);

template <typename K>
size_t sort_workspace_bytes(long long n);

// Stable sort of (key, value) pairs by key bits [begin_bit, end_bit). keys_in/vals_in are not
// modified; results land in keys_out/vals_out (which must not alias the inputs). With gather_out
// (device, n entries), the last pass also writes gather_out[i] = gather_table[vals_out[i]].
// With n_dev (device), n is a capacity: the pairs sorted are the first min(*n_dev, n), a count that
// the host never reads; the launches are sized for n.
template <typename K>
int radix_sort_pairs(const K* keys_in, const uint32_t* vals_in, K* keys_out, uint32_t* vals_out,
                     long long n, int begin_bit, int end_bit, void* ws, size_t ws_bytes,
                     cudaStream_t stream, const uint32_t* gather_table = nullptr,
                     uint32_t* gather_out = nullptr, const uint32_t* n_dev = nullptr);

// Number of significant bits needed to represent v (0 for v == 0).
inline int bit_width(unsigned long long v) {
    int b = 0;
    while (v) {
        ++b;
        v >>= 1;
    }
    return b;
}

}  // namespace splat
