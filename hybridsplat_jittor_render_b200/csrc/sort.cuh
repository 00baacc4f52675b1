// Device-wide stable LSD radix sort of (uint32 key, uint32 value) pairs and
// the decoupled look-back primitive it shares with the pair-offset scan
// (binning.cuh).
//
// These replace the reference's CUB calls (vendor/flashgs/cuda_rasterizer/
// sort.cu:29-58, rasterizer/full_rasterizer.cu:301-355). Only the ordering
// contract matters for parity: the sort is stable, so equal keys keep their
// input order, and the scan is exact integer arithmetic.
//
// The sort is a "onesweep" LSD radix sort (Adinets and Merrill, 2022): one
// histogram kernel computes the digit counts of every pass in a single read
// of the keys, then each 8-bit pass is ONE kernel in which every block ranks
// its tile in shared memory, obtains the counts of all earlier tiles by
// decoupled look-back and scatters its items digit-run by digit-run.
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
constexpr int kMaxPasses = 4;                        // 32-bit keys

// Look-back status words: two flag bits over a 30-bit count.
constexpr uint32_t kFlagAggregate = 1u << 30;
constexpr uint32_t kFlagInclusive = 2u << 30;
constexpr uint32_t kValueMask = (1u << 30) - 1u;
constexpr uint32_t kMaxItems = kValueMask;           // counts must fit 30 bits

// Every wait of the sort and scan kernels (a look-back on a predecessor's
// status word, the tile's bulk copy) is bounded. A predecessor tile is always
// resident (tiles are numbered in the order blocks start), so a wait in a
// correct launch ends within microseconds; a wait still unanswered after
// kWaitLimitNs of device time (%globaltimer), or after kSpinLimit polls
// should the timer not advance, gives up: it sets bit 0 of the caller's error
// word and returns. Every kernel that consumes a sort or scan result reads
// that word first and does nothing when it is set, so a give-up never turns
// into out-of-range indices downstream; the raster call reports it as an
// error of the same call.
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s
constexpr uint32_t kSpinLimit = 1u << 28;

// Test hook value: no tile stalls.
constexpr uint32_t kNoStall = 0xffffffffu;

inline uint32_t tiles_for(uint32_t count) { return (count + kTile - 1) / kTile; }

// Scratch bytes needed by sort_pairs for `count` items.
uint64_t sort_scratch_bytes(uint32_t count);

// Key of an item that a dropping sort leaves out (see sort_pairs' kept).
constexpr uint32_t kDropKey = 0xffffffffu;

// Stable sort of keys[0, count) by bits [begin_bit, end_bit) of the key.
// keys/vals hold the input and receive the output; alt_keys/alt_vals are
// ping-pong buffers of the same size. scratch holds sort_scratch_bytes(count)
// bytes; error (may be null) receives bit 0 if a wait gave up, and when it is
// already set on entry every pass does nothing. stall_tile is a test hook:
// the block of that tile in the first pass never publishes its look-back
// status, so the waits of its successors run out (kNoStall: none).
// kept (device word, may be null; full 32-bit sorts only): the items whose
// key is kDropKey are left out. *kept, written by an earlier kernel of the
// stream, must be the number of the other items; they are sorted into
// keys/vals[0, *kept) in the same stable order, and the passes after the
// first only touch those. The depth sorts use it to skip the Gaussians that
// emit no pair.
// bound (device word, may be null; not with kept): every pass sorts only the
// first min(*bound, count) items, so `count` may be a capacity that sizes the
// grids and *bound the number of items an earlier kernel of the stream
// wrote. The launches then depend on the capacity alone (a captured graph
// replays them for any item count up to it).
// Launches: one memset, one histogram kernel, one kernel per 8-bit pass
// (plus two copies when the pass count is odd).
cudaError_t sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals,
                       uint32_t count, int begin_bit, int end_bit, void* scratch,
                       cudaStream_t stream, uint32_t* error = nullptr,
                       uint32_t stall_tile = kNoStall, const uint32_t* kept = nullptr,
                       const uint32_t* bound = nullptr);

// Number of bits needed to hold values in [0, n): the reference's
// getHigherMsb(n) for the tile count (sort.cu:141-156).
inline int bits_for_tiles(uint32_t n) {
    int bits = 0;
    while (bits < 32 && (n >> bits) != 0u) ++bits;
    return bits;
}

// ---- device helpers shared with the fused scan-and-emit kernels ----

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Poll counter of one bounded wait: expired() is called once per
// unsuccessful poll and turns true when the wait must give up.
struct WaitClock {
    uint64_t start = 0;
    uint32_t polls = 0;
    __device__ __forceinline__ bool expired() {
        if (++polls > kSpinLimit) return true;
        if ((polls & 31u) != 1u) return false;
        const uint64_t now = global_ns();
        if (start == 0) start = now;
        return now - start > kWaitLimitNs;
    }
};

// True when a bounded wait of this call has given up: the error word is
// written by earlier kernels of the same stream (visible at kernel start) or
// by other blocks of the running kernel.
__device__ __forceinline__ bool wait_failed(const uint32_t* error) {
    return error != nullptr && *reinterpret_cast<const volatile uint32_t*>(error) != 0u;
}

__device__ __forceinline__ uint32_t load_status(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void store_status(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Exclusive prefix of `status[tile * stride]` over all earlier tiles, by
// decoupled look-back. The caller has already published its own aggregate.
// kWindow predecessors are read per step, so a chain of tiles that have only
// published aggregates costs one memory round trip per kWindow tiles.
constexpr int kLookBackWindow = 8;

template <int kWindow = kLookBackWindow>
__device__ __forceinline__ uint32_t look_back(const uint32_t* status, uint32_t tile,
                                              uint32_t stride, uint32_t* error) {
    uint32_t prefix = 0;
    int64_t t = static_cast<int64_t>(tile) - 1;
    WaitClock clock;
    while (t >= 0) {
        uint32_t s[kWindow];
#pragma unroll
        for (int k = 0; k < kWindow; ++k) {
            s[k] = t - k >= 0 ? load_status(status + static_cast<uint64_t>(t - k) * stride)
                              : kFlagInclusive;
        }
        int k = 0;
#pragma unroll
        for (int i = 0; i < kWindow; ++i) {
            if (k != i || (s[i] & ~kValueMask) == 0u) continue;  // stopped, or not published yet
            prefix += s[i] & kValueMask;
            if ((s[i] & kFlagInclusive) != 0u) return prefix;
            k = i + 1;
        }
        if (k == 0) {
            if (clock.expired()) {
                if (error != nullptr) atomicOr(error, 1u);
                return prefix;
            }
            __nanosleep(32);
        }
        t -= k;
    }
    return prefix;
}

}  // namespace sort
}  // namespace hs
