// Device-wide stable LSD radix sort of (uint32 key, uint32 value) pairs and
// an exclusive scan of uint32 counts.
//
// These replace the reference's CUB calls (vendor/flashgs/cuda_rasterizer/
// sort.cu:29-58, rasterizer/full_rasterizer.cu:301-355). Only the ordering
// contract matters for parity: the sort is stable, so equal keys keep their
// input order, and the scan is exact integer arithmetic.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hs {
namespace sort {

constexpr int kThreads = 256;                        // 8 warps
constexpr int kItemsPerThread = 8;
constexpr int kTile = kThreads * kItemsPerThread;    // 2048 items per block
constexpr int kRadixBits = 8;
constexpr int kBins = 1 << kRadixBits;

inline uint32_t tiles_for(uint32_t count) { return (count + kTile - 1) / kTile; }

// Scratch bytes needed by sort_pairs / exclusive_scan for `count` items.
uint64_t sort_scratch_bytes(uint32_t count);
uint64_t scan_scratch_bytes(uint32_t count);

// Stable sort of keys[0, count) by bits [begin_bit, end_bit) of the key.
// keys/vals hold the input and receive the output; alt_keys/alt_vals are
// ping-pong buffers of the same size. scratch holds sort_scratch_bytes(count).
cudaError_t sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals,
                       uint32_t count, int begin_bit, int end_bit, void* scratch,
                       cudaStream_t stream);

// out[i] = sum(in[gather[j]] for j < i) when gather != nullptr, else
// sum(in[j] for j < i); *total = the full sum. out may alias in when
// gather == nullptr (each thread reads its items before writing them).
cudaError_t exclusive_scan(const uint32_t* in, const uint32_t* gather, uint32_t* out,
                           uint32_t* total, uint32_t count, void* scratch, cudaStream_t stream);

// Number of bits needed to hold values in [0, n): the reference's
// getHigherMsb(n) for the tile count (sort.cu:141-156).
inline int bits_for_tiles(uint32_t n) {
    int bits = 0;
    while (bits < 32 && (n >> bits) != 0u) ++bits;
    return bits;
}

}  // namespace sort
}  // namespace hs
