// Pair emission and tile ranges shared by both backends.
//
// After the depth sort, `order` lists the Gaussians by (depth bits, index).
// offsets_kernel scans the per-Gaussian pair counts in that order (a
// single-pass exclusive scan with decoupled look-back across blocks) and
// stores each Gaussian's first pair slot by Gaussian index.
// emit_flat_compact_kernel then writes the pairs, walking the Gaussians in
// index order so that the large
// screen-space footprints of the nearest Gaussians (adjacent in depth order)
// spread over all blocks. Pairs of one Gaussian may be written in any order
// among themselves: each names a different tile, and the following stable
// sort by tile id keeps, for every tile, the depth order of the Gaussians.
// The result is the reference's lexicographic (tile | depth key, index)
// order (vendor/flashgs/cuda_rasterizer/sort.cu:160-189,
// rasterizer/full_rasterizer.cu:127-153).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "sort.cuh"

namespace hs {
namespace bin {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 8;                          // sorted positions per thread
constexpr int kScanTile = kScanThreads * kScanItems;   // 2048 Gaussians per block
constexpr int kEmitThreads = 256;

inline uint32_t scan_tiles(uint32_t count) { return (count + kScanTile - 1) / kScanTile; }

// Publishes the four totals words of a raster call to mapped pinned host
// memory from the SMs. A cudaMemcpyAsync of them would queue on the
// device-to-host copy engine behind any bulk read-back the caller has in
// flight (a previous frame's maps), delaying the host's wait for the pair
// count by the whole transfer; stores from a kernel do not.
static __global__ void publish_totals_kernel(const uint32_t* __restrict__ totals,
                                             volatile uint32_t* host) {
    if (threadIdx.x < 4) host[threadIdx.x] = totals[threadIdx.x];
    __threadfence_system();
}

// The status of the raster calls of one graph replay, for the host: per call
// (blockIdx.x) its first three totals words (rendered, prefiltered
// violation, emitted pairs) and its wait-status word, to the call's mapped
// totals block. Launched on a branch of the graph that follows every call's
// binning, so that no renderer waits for these stores to reach the host.
struct ViewStatusCall {
    const uint32_t* totals;
    const uint32_t* error;
    volatile uint32_t* host;
};
struct ViewStatusArgs {
    ViewStatusCall call[2];
};
static __global__ void view_status_kernel(ViewStatusArgs a) {
    const ViewStatusCall c = a.call[blockIdx.x];
    if (threadIdx.x < 3) c.host[threadIdx.x] = c.totals[threadIdx.x];
    if (threadIdx.x == 3) c.host[3] = *reinterpret_cast<const volatile uint32_t*>(c.error);
    __threadfence_system();
}

// Allocates the mapped pinned totals block of a context: *host for the host,
// *device for kernels.
inline cudaError_t alloc_mapped_totals(uint32_t** host, uint32_t** device) {
    cudaError_t st = cudaHostAlloc(reinterpret_cast<void**>(host), 4 * sizeof(uint32_t),
                                   cudaHostAllocPortable | cudaHostAllocMapped);
    if (st != cudaSuccess) return st;
    st = cudaHostGetDevicePointer(reinterpret_cast<void**>(device), *host, 0);
    if (st != cudaSuccess) {
        cudaFreeHost(*host);
        *host = nullptr;
    }
    return st;
}
// Scratch words of offsets_kernel (counter + one status word per block);
// zeroed before the launch.
inline uint64_t scan_scratch_bytes(uint32_t count) {
    return (static_cast<uint64_t>(scan_tiles(count > 0 ? count : 1)) + 64) * sizeof(uint32_t);
}

// The next pair slot of Gaussian `owner` for the calling lane. The lanes of
// the warp that take a slot of the same Gaussian at this call share one
// shared-memory atomic (the leader fetches the base for all of them, each adds
// its rank among them) instead of issuing one atomic each on the same address,
// which the hardware serialises. Slots of one Gaussian are handed out in some
// order either way: its pairs name different tiles, and the stable tile sort
// that follows makes their order irrelevant.
__device__ __forceinline__ uint32_t take_slot(uint32_t* cursor, uint32_t owner) {
    const uint32_t active = __activemask();
    const uint32_t peers = __match_any_sync(active, owner);
    const int lane = threadIdx.x & 31;
    const int leader = __ffs(peers) - 1;
    uint32_t first = 0;
    if (lane == leader) first = atomicAdd(&cursor[owner], static_cast<uint32_t>(__popc(peers)));
    first = __shfl_sync(peers, first, leader);
    return first + static_cast<uint32_t>(__popc(peers & ((1u << lane) - 1u)));
}

__device__ __forceinline__ uint32_t warp_sum(uint32_t v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// first_pair[order[i]] = sum(counts[order[j]] for j < i), for i below
// *live_count (the Gaussians a dropping depth sort kept) or, when live_count
// is null, below count. The grid covers count; blocks past the live items leave.
static __global__ void __launch_bounds__(kScanThreads) offsets_kernel(
    uint32_t count, const uint32_t* __restrict__ live_count, const uint32_t* __restrict__ order,
    const uint32_t* __restrict__ counts, uint32_t* __restrict__ control,
    uint32_t* __restrict__ error, uint32_t* __restrict__ first_pair) {
    __shared__ uint32_t warp_sums[kScanThreads / 32];
    __shared__ uint32_t tile_slot, tile_prefix;
    uint32_t* counter = control;
    uint32_t* status = control + 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (sort::wait_failed(error)) return;  // the depth order is not a permutation
    if (threadIdx.x == 0) tile_slot = atomicAdd(counter, 1u);
    __syncthreads();
    const uint32_t tile = tile_slot;
    if (live_count != nullptr) count = *live_count;
    if (static_cast<uint64_t>(tile) * kScanTile >= count) return;  // no block waits on a later tile
    const uint64_t base = static_cast<uint64_t>(tile) * kScanTile +
                          static_cast<uint64_t>(threadIdx.x) * kScanItems;
    uint32_t gid[kScanItems], cnt[kScanItems];
    uint32_t local = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const uint64_t i = base + k;
        gid[k] = i < count ? order[i] : 0u;
        cnt[k] = i < count ? counts[gid[k]] : 0u;
        local += cnt[k];
    }
    uint32_t incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t sum = 0;
        for (int w = 0; w < kScanThreads / 32; ++w) sum += warp_sums[w];
        uint32_t earlier = 0;
        if (tile == 0) {
            sort::store_status(status, sort::kFlagInclusive | (sum & sort::kValueMask));
        } else {
            sort::store_status(status + tile, sort::kFlagAggregate | (sum & sort::kValueMask));
            earlier = sort::look_back(status, tile, 1, error);
            sort::store_status(status + tile,
                               sort::kFlagInclusive | ((earlier + sum) & sort::kValueMask));
        }
        tile_prefix = earlier;
    }
    __syncthreads();
    uint32_t run = tile_prefix;
    for (int w = 0; w < warp; ++w) run += warp_sums[w];
    run += incl - local;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        if (cnt[k] != 0u) first_pair[gid[k]] = run;
        run += cnt[k];
    }
}

// Per-tile [start, end) of the sorted pair list. Entries of tiles without
// pairs keep the zeros written before the launch. Tile ids >= tile_count are
// padding and are ignored. Each thread reads four consecutive tile ids with
// one 16-byte load (the arrays are 16-byte aligned) plus the id before them;
// the grid strides over the list (ranges_grid blocks of kRangeThreads).
constexpr int kRangeThreads = 256;

inline unsigned ranges_grid(uint32_t pair_count) {
    const uint64_t quads = (static_cast<uint64_t>(pair_count) + 3) / 4;
    const uint64_t blocks = (quads + kRangeThreads - 1) / kRangeThreads;
    return static_cast<unsigned>(blocks < 148 * 8 ? (blocks > 0 ? blocks : 1) : 148 * 8);
}

// bound (device word, may be null): only the first min(*bound, pair_count)
// pairs are read, for a grid sized by a capacity.
template <class Range>
__global__ void __launch_bounds__(kRangeThreads) ranges_kernel(
    uint32_t pair_count, uint32_t tile_count, const uint32_t* __restrict__ tile_ids,
    Range* __restrict__ ranges, const uint32_t* __restrict__ bound = nullptr) {
    using Index = decltype(ranges[0].x);
    if (bound != nullptr) pair_count = min(*bound, pair_count);
    const uint32_t quads = (pair_count + 3u) / 4u;
    for (uint32_t q = blockIdx.x * kRangeThreads + threadIdx.x; q < quads;
         q += gridDim.x * kRangeThreads) {
        const uint32_t base = q * 4u;
        uint32_t t[4];
        if (base + 4u <= pair_count) {
            const uint4 v = reinterpret_cast<const uint4*>(tile_ids)[q];
            t[0] = v.x;
            t[1] = v.y;
            t[2] = v.z;
            t[3] = v.w;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) t[k] = base + k < pair_count ? tile_ids[base + k] : 0u;
        }
        uint32_t prev = base == 0u ? 0xffffffffu : tile_ids[base - 1u];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t i = base + k;
            if (i >= pair_count) break;
            if (t[k] != prev) {
                if (t[k] < tile_count) ranges[t[k]].x = static_cast<Index>(i);
                if (prev < tile_count) ranges[prev].y = static_cast<Index>(i);
            }
            if (i == pair_count - 1u && t[k] < tile_count) ranges[t[k]].y = static_cast<Index>(pair_count);
            prev = t[k];
        }
    }
}

// Flattened emission for emitters that keep a subset of a rectangle (the
// FlashGS tile/ellipse test): the rectangle tiles of a warp's 32 Gaussians
// are dealt to the lanes round-robin, and a kept tile takes the next slot of
// its Gaussian from a shared-memory cursor. Slots of one Gaussian are thus
// filled in no particular order, which the following stable sort by tile id
// makes irrelevant (each tile appears once per Gaussian).
// Emitter interface: Shape, load(gid), and
//   __device__ uint32_t slots(const Shape&) const;             // rectangle size
//   struct Cache;                                               // per-lane scratch, value-initialised
//   __device__ bool pair_at(const Shape&, uint32_t owner, uint32_t k, uint32_t& tile,
//                           uint32_t& tag, Cache&) const;        // kept? tile, value bits
// `owner` names the Gaussian within the block, so an emitter may keep work
// shared by consecutive pairs of one Gaussian in its Cache.
// The value of a kept pair is the Gaussian index | tag. A Gaussian never
// writes more than its counted pairs. Nothing is written when a bounded wait
// of the call has given up (first_pair is then not a valid offset table).
template <class Emitter>
__global__ void __launch_bounds__(kEmitThreads) emit_flat_compact_kernel(
    uint32_t count, const uint32_t* __restrict__ counts, const uint32_t* __restrict__ first_pair,
    Emitter em, uint32_t* __restrict__ tile_ids, uint32_t* __restrict__ values,
    const uint32_t* __restrict__ error) {
    if (sort::wait_failed(error)) return;
    __shared__ typename Emitter::Shape shapes[kEmitThreads];
    __shared__ uint32_t offsets[kEmitThreads], inclusive[kEmitThreads], cursor[kEmitThreads],
        counted[kEmitThreads];
    const uint32_t gid = blockIdx.x * kEmitThreads + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const uint32_t base = threadIdx.x & ~31u;
    const uint32_t cnt = gid < count ? counts[gid] : 0u;
    const typename Emitter::Shape mine = em.load(cnt != 0u ? gid : 0u);
    shapes[threadIdx.x] = mine;
    offsets[threadIdx.x] = cnt != 0u ? first_pair[gid] : 0u;
    cursor[threadIdx.x] = 0;
    counted[threadIdx.x] = cnt;
    uint32_t incl = cnt != 0u ? em.slots(mine) : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    inclusive[threadIdx.x] = incl;
    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
    __syncwarp();
    typename Emitter::Cache cache{};
    for (uint32_t f = lane; f < total; f += 32) {
        uint32_t j = 0;
#pragma unroll
        for (uint32_t step = 16; step >= 1; step >>= 1) {
            if (inclusive[base + j + step - 1] <= f) j += step;
        }
        const uint32_t owner = base + j;
        const uint32_t k = f - (j == 0 ? 0u : inclusive[owner - 1]);
        uint32_t tile, tag = 0;
        if (em.pair_at(shapes[owner], owner, k, tile, tag, cache)) {
            const uint32_t slot = take_slot(cursor, owner);
            if (slot < counted[owner]) {
                tile_ids[offsets[owner] + slot] = tile;
                values[offsets[owner] + slot] = (blockIdx.x * kEmitThreads + owner) | tag;
            }
        }
    }
}

// Rasterisation order of the tiles: longest pair lists first (buckets of an
// eighth of an octave of the list length: its bit length and the three bits
// below the leading one; any order inside a bucket), so that the persistent
// rasterisers take the expensive tiles before the cheap ones.
// One block of kOrderThreads threads over tiles [tile_first, tile_first +
// tile_count); `counter` (the rasteriser's work counter) is reset here. When
// host_error (mapped pinned memory) is given, the call's look-back error word
// (set when a bounded wait of its depth sort, pair-offset scan or tile sort
// gave up) is published to it: this is the last kernel of binning, the host
// reads the word once binning is done and fails the same call.
constexpr int kOrderThreads = 1024;

template <class Range>
__global__ void __launch_bounds__(kOrderThreads) tile_order_kernel(
    uint32_t tile_first, uint32_t tile_count, const Range* __restrict__ ranges,
    uint32_t* __restrict__ order, uint32_t* __restrict__ counter, const uint32_t* __restrict__ error,
    volatile uint32_t* host_error) {
    constexpr uint32_t kBuckets = 33u * 8u;
    constexpr uint32_t kScanWarps = (kBuckets + 31u) / 32u;
    static_assert(kScanWarps <= 32u && kScanWarps * 32u <= static_cast<uint32_t>(kOrderThreads), "scan");
    __shared__ uint32_t hist[kBuckets];
    __shared__ uint32_t next[kBuckets];
    __shared__ uint32_t warp_base[kScanWarps];
    // bucket 8 * clz + (7 - next three bits): ascending buckets, descending lengths
    auto bucket = [](uint32_t len) -> uint32_t {
        if (len == 0u) return kBuckets - 1u;
        const uint32_t lz = __clz(len);
        return lz * 8u + (7u - (((len << lz) << 1) >> 29));
    };
    for (uint32_t b = threadIdx.x; b < kBuckets; b += kOrderThreads) hist[b] = 0;
    if (threadIdx.x == 0) *counter = 0;
    __syncthreads();
    for (uint32_t t = tile_first + threadIdx.x; t < tile_first + tile_count; t += kOrderThreads) {
        const uint32_t len = static_cast<uint32_t>(ranges[t].y - ranges[t].x);
        atomicAdd(&hist[bucket(len)], 1u);
    }
    __syncthreads();
    // exclusive scan of the bucket counts: one warp-level scan per 32 buckets,
    // then a scan of the warps' totals
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t count = 0, incl = 0;
    if (warp < kScanWarps) {
        count = threadIdx.x < kBuckets ? hist[threadIdx.x] : 0u;
        incl = count;
#pragma unroll
        for (uint32_t off = 1; off < 32u; off <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += t;
        }
        if (lane == 31u) warp_base[warp] = incl;
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t total = lane < kScanWarps ? warp_base[lane] : 0u;
        uint32_t run = total;
#pragma unroll
        for (uint32_t off = 1; off < 32u; off <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, run, off);
            if (lane >= off) run += t;
        }
        __syncwarp();
        if (lane < kScanWarps) warp_base[lane] = run - total;
    }
    __syncthreads();
    if (warp < kScanWarps && threadIdx.x < kBuckets) next[threadIdx.x] = warp_base[warp] + incl - count;
    __syncthreads();
    for (uint32_t t = tile_first + threadIdx.x; t < tile_first + tile_count; t += kOrderThreads) {
        const uint32_t len = static_cast<uint32_t>(ranges[t].y - ranges[t].x);
        order[atomicAdd(&next[bucket(len)], 1u)] = t;
    }
    if (host_error != nullptr && threadIdx.x == 0) {
        host_error[0] = *reinterpret_cast<const volatile uint32_t*>(error);
        __threadfence_system();
    }
}

}  // namespace bin
}  // namespace hs
