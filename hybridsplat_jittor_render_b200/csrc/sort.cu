// Stable LSD radix sort (sort.cuh), 8-bit digits, in one of two pass forms.
//
// Onesweep (below 2M items). Scratch (zeroed by one memset per sort):
//   hist[kMaxPasses][kBins]          digit counts of every pass
//   tile_counter[kMaxPasses]         dynamic tile numbering per pass
//   status[kMaxPasses][tiles][kBins] look-back words
// One histogram kernel reads the keys once for all passes; then each pass is
// one kernel whose blocks
//   1. take the next tile number (so every earlier tile's block has already
//      started and will publish without waiting on this one) and copy the
//      tile's keys and values into shared memory with two bulk asynchronous
//      copies (the TMA engine; a ragged tail of < 4 items with plain loads),
//      so no thread holds the items in registers while ranking;
//   2. rank the tile stably: warp w owns a contiguous segment and walks it 32
//      items at a time, grouping equal digits with __match_any_sync (or one
//      ballot per digit bit); per-warp digit counts are prefixed across warps;
//   3. publish their per-digit counts, look back for the counts of all earlier
//      tiles and publish the inclusive sums;
//   4. permute the tile in shared memory into digit order and write each
//      digit run to consecutive global positions (coalesced).
// Keeping the tile in shared memory instead of registers lets several blocks
// share an SM, which hides the latency of the look-back.
//
// Reduce-then-scan (from 2M items). Scratch: counts[kBins][tiles], totals.
// Each pass is a count kernel (per 4096-item tile, the digit counts), a scan
// kernel (per digit, the exclusive prefix across tiles and the total) and a
// scatter kernel whose blocks do steps 1, 2 and 4 with the destination of each
// digit run read from the scan: no block waits on another. When all resident
// blocks start together, a onesweep tile walks back over many predecessors
// that have only published their aggregate; at these sizes that walk cost more
// than the two extra launches.
#include <utility>

#include "sort.cuh"

namespace hs {
namespace sort {
namespace {

constexpr int kWarps = kThreads / 32;

// Pass kernels come in two tile sizes: 2048 items (8 per thread) below 256K
// items, 4096 items (16 per thread) from there on. Larger tiles halve the rate
// at which tiles start, and with it the number of predecessors a new tile
// finds holding only an aggregate; the look-back of the large variant also
// reads more of them per round trip. Within a warp, items are ranked either
// with __match_any_sync or with one ballot per digit bit; ballots measured
// faster for full-width (four-pass) keys and for sorts of 8M items or more,
// MATCH for the two-pass tile sorts below that.
constexpr int kLargeItems = 16;
constexpr int kLargeWindow = 16;
constexpr uint32_t kLargeTileItems = 1u << 18;
constexpr uint32_t kBallotItems = 1u << 23;
// From 2M items a pass is three kernels (count, scan across tiles, scatter)
// instead of one with a decoupled look-back: measured on a B200, 3.66M 13-bit
// keys 124 -> 109 us and 30M 15-bit keys 620 -> 487 us, while below about 1M
// items the extra launches cost more than the look-back.
constexpr uint32_t kSplitItems = 1u << 21;

struct SortScratch {
    uint32_t* hist;       // [kMaxPasses][kBins]
    uint32_t* counters;   // [kMaxPasses]
    uint32_t* status;     // [kMaxPasses][tiles][kBins]
    uint64_t zero_bytes;  // bytes to clear before the sort
};

SortScratch sort_scratch(void* base, uint32_t tiles, int passes) {
    SortScratch s;
    s.hist = static_cast<uint32_t*>(base);
    s.counters = s.hist + kMaxPasses * kBins;
    s.status = s.counters + 64;  // keep status 256-byte aligned
    s.zero_bytes = (static_cast<uint64_t>(kMaxPasses) * kBins + 64 +
                    static_cast<uint64_t>(passes) * tiles * kBins) *
                   sizeof(uint32_t);
    return s;
}

__device__ __forceinline__ uint32_t digit_of(uint32_t key, int shift, uint32_t mask) {
    return (key >> shift) & mask;
}

// Digit counts of every pass in one read of the keys: 16-byte loads (the key
// arrays are 16-byte aligned), per-block shared-memory counts.
__global__ void __launch_bounds__(kThreads) histogram_kernel(const uint32_t* __restrict__ keys,
                                                             uint32_t count, int begin_bit,
                                                             int end_bit, int drop,
                                                             uint32_t* __restrict__ hist,
                                                             const uint32_t* __restrict__ bound) {
    __shared__ uint32_t bins[kMaxPasses][kBins];
    if (bound != nullptr) count = min(*bound, count);
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    for (int p = 0; p < passes; ++p) bins[p][threadIdx.x] = 0;
    __syncthreads();
    auto count_key = [&](uint32_t key) {
        if (drop && key == kDropKey) return;  // left out of a dropping sort
        for (int p = 0; p < passes; ++p) {
            const int shift = begin_bit + p * kRadixBits;
            const int bits = min(kRadixBits, end_bit - shift);
            atomicAdd(&bins[p][digit_of(key, shift, (1u << bits) - 1u)], 1u);
        }
    };
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    const uint64_t quads = count / 4u;
    const uint4* keys4 = reinterpret_cast<const uint4*>(keys);
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < quads;
         i += stride) {
        const uint4 q = keys4[i];
        count_key(q.x);
        count_key(q.y);
        count_key(q.z);
        count_key(q.w);
    }
    if (blockIdx.x == 0 && threadIdx.x < count - quads * 4u) count_key(keys[quads * 4u + threadIdx.x]);
    __syncthreads();
    for (int p = 0; p < passes; ++p) {
        const uint32_t v = bins[p][threadIdx.x];
        if (v != 0u) atomicAdd(&hist[p * kBins + threadIdx.x], v);
    }
}

__device__ __forceinline__ uint32_t shared_address(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Bulk asynchronous copy global -> shared, completing on an mbarrier. Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* barrier) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(shared_address(dst)), "l"(src), "r"(bytes), "r"(shared_address(barrier))
        : "memory");
}

__device__ __forceinline__ bool barrier_try_wait(uint64_t* barrier, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(shared_address(barrier)), "r"(parity)
        : "memory");
    return done != 0u;
}

// Bounded wait for phase 0 of the tile barrier; false when it gave up.
__device__ __forceinline__ bool wait_tile(uint64_t* barrier) {
    WaitClock clock;
    while (!barrier_try_wait(barrier, 0u)) {
        if (clock.expired()) return false;
    }
    return true;
}

// Exclusive scan of 256 values held one per thread (all kThreads threads).
__device__ __forceinline__ uint32_t block_exclusive_256(uint32_t v, uint32_t* warp_sums) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += t;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    uint32_t base = 0;
    for (int w = 0; w < warp; ++w) base += warp_sums[w];
    __syncthreads();
    return base + incl - v;
}

// ---- the tile of one pass block, shared by both pass forms ----

template <int kItems>
struct PassTile {
    static constexpr uint32_t kTileItems = kThreads * kItems;
    // The tile, in input order until it is permuted into digit order.
    alignas(16) uint32_t keys[kTileItems];
    alignas(16) uint32_t vals[kTileItems];
    uint32_t warp_count[kWarps][kBins];
    uint32_t digit_start[kBins];   // first local position of each digit
    uint32_t global_base[kBins];   // destination of the digit run's first item
    uint32_t warp_sums[kWarps];
    uint32_t slot;
    uint32_t kept;                 // items of the tile that are written
    alignas(8) uint64_t loaded;    // completes when the bulk copies land
};

// Barrier set-up and per-warp digit counts cleared; ends with a block barrier.
template <int kItems>
__device__ __forceinline__ void tile_begin(PassTile<kItems>& t) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(shared_address(&t.loaded))
                     : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int b = lane; b < kBins; b += 32) t.warp_count[warp][b] = 0;
    __syncthreads();
}

// Copies keys/values [begin, begin + n) into the tile: whole 16-byte groups
// with two bulk asynchronous copies (the TMA engine), a ragged tail of < 4
// items with plain loads.
template <int kItems>
__device__ __forceinline__ void tile_issue_load(PassTile<kItems>& t, const uint32_t* keys_in,
                                                const uint32_t* vals_in, uint64_t begin, uint32_t n) {
    const uint32_t bulk = n & ~3u;
    if (threadIdx.x == 0) {
        if (bulk != 0u) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                         ::"r"(shared_address(&t.loaded)), "r"(2u * bulk * 4u) : "memory");
            bulk_load(t.keys, keys_in + begin, bulk * 4u, &t.loaded);
            bulk_load(t.vals, vals_in + begin, bulk * 4u, &t.loaded);
        } else {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                         ::"r"(shared_address(&t.loaded)) : "memory");
        }
    }
    if (threadIdx.x < n - bulk) {
        t.keys[bulk + threadIdx.x] = keys_in[begin + bulk + threadIdx.x];
        t.vals[bulk + threadIdx.x] = vals_in[begin + bulk + threadIdx.x];
    }
}

// Waits (bounded) for the tile's copies; false, with the error reported, when
// the wait gave up (the block must then leave).
template <int kItems>
__device__ __forceinline__ bool tile_wait_load(PassTile<kItems>& t, uint32_t* error) {
    const bool landed = wait_tile(&t.loaded);
    if (!__syncthreads_and(landed)) {
        // The copies did not complete within the bound: report, wait once more
        // (bounded) so that no copy is left writing this block's shared memory.
        if (threadIdx.x == 0) {
            if (error != nullptr) atomicOr(error, 1u);
            wait_tile(&t.loaded);
        }
        return false;
    }
    return true;
}

// Stable ranking of the tile's n items by digit: warp w owns the contiguous
// segment [w kItems 32, (w + 1) kItems 32) and walks it 32 items at a time,
// grouping equal digits with __match_any_sync or one ballot per digit bit.
// On return rank[] holds each item's position among equal digits of its
// warp's earlier items, warp_count[w][d] the exclusive prefix of warp w for
// digit d, and the result is this thread's digit's (threadIdx.x) tile total.
// Dropped items (drop and key == kDropKey) take no rank.
template <int kItems, bool kBallot>
__device__ __forceinline__ uint32_t tile_rank(PassTile<kItems>& t, uint32_t n, int drop, int shift,
                                              int bits, uint32_t (&rank)[kItems]) {
    constexpr uint32_t kWarpItems = PassTile<kItems>::kTileItems / kWarps;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t seg = static_cast<uint32_t>(warp) * kWarpItems;
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = seg + static_cast<uint32_t>(k) * 32u + lane;
        const uint32_t key = i < n ? t.keys[i] : 0u;
        const bool valid = i < n && !(drop && key == kDropKey);
        const uint32_t dg = valid ? digit_of(key, shift, mask) : 0u;
        uint32_t peers;
        if (kBallot) {
            // lanes holding the same digit, one ballot per digit bit (cheaper
            // than __match_any_sync when many blocks share an SM)
            peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
            for (int bit = 0; bit < kRadixBits; ++bit) {
                if (bit < bits) {
                    const uint32_t set = (dg >> bit) & 1u;
                    const uint32_t vote = __ballot_sync(0xffffffffu, set != 0u);
                    peers &= set != 0u ? vote : ~vote;
                }
            }
        } else {
            peers = __match_any_sync(0xffffffffu, valid ? static_cast<int>(dg) : -1);
        }
        const int dig = valid ? static_cast<int>(dg) : -1;
        const uint32_t before = dig >= 0 ? t.warp_count[warp][dig] : 0u;
        __syncwarp();
        rank[k] = before + __popc(peers & lt_mask);
        const int leader = __ffs(peers) - 1;
        if (dig >= 0 && lane == leader) t.warp_count[warp][dig] = before + __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    // per-digit totals of the tile and the exclusive per-warp prefixes
    const int b = threadIdx.x;
    uint32_t total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const uint32_t c = t.warp_count[w][b];
        t.warp_count[w][b] = total;
        total += c;
    }
    return total;
}

// With global_base[] set for every digit: the tile's digit starts from the
// totals, the tile permuted in place into digit order (keys, then values),
// each digit run written to consecutive global positions.
template <int kItems>
__device__ __forceinline__ void tile_scatter(PassTile<kItems>& t, uint32_t n, int drop, int shift,
                                             int bits, uint32_t total, uint32_t (&rank)[kItems],
                                             uint32_t* keys_out, uint32_t* vals_out) {
    constexpr uint32_t kWarpItems = PassTile<kItems>::kTileItems / kWarps;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t seg = static_cast<uint32_t>(warp) * kWarpItems;
    const int b = threadIdx.x;
    const uint32_t local_start = block_exclusive_256(total, t.warp_sums);
    t.digit_start[b] = local_start;
    if (b == kBins - 1) t.kept = local_start + total;
    uint32_t item[kItems];
    bool keep[kItems];
    __syncthreads();  // digit_start, global_base
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = seg + static_cast<uint32_t>(k) * 32u + lane;
        item[k] = t.keys[i];
        keep[k] = i < n && !(drop && item[k] == kDropKey);
        if (keep[k]) {
            const uint32_t d = digit_of(item[k], shift, mask);
            rank[k] += t.digit_start[d] + t.warp_count[warp][d];  // final position in the tile
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        if (keep[k]) t.keys[rank[k]] = item[k];
    }
#pragma unroll
    for (int k = 0; k < kItems; ++k) item[k] = t.vals[seg + static_cast<uint32_t>(k) * 32u + lane];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        if (keep[k]) t.vals[rank[k]] = item[k];
    }
    __syncthreads();
    const uint32_t written = t.kept;  // n unless the pass drops items
    for (uint32_t i = threadIdx.x; i < written; i += kThreads) {
        const uint32_t k = t.keys[i];
        const uint32_t d = digit_of(k, shift, mask);
        const uint32_t dst = t.global_base[d] + (i - t.digit_start[d]);
        keys_out[dst] = k;
        vals_out[dst] = t.vals[i];
    }
}

// Items of a pass: *live_count (the survivors after a dropping first pass, or
// the bound of a sort sized for a capacity), at most count; else count.
__device__ __forceinline__ uint32_t pass_items(uint32_t count, const uint32_t* live_count) {
    return live_count != nullptr ? min(*live_count, count) : count;
}

// ---- onesweep pass: one kernel, cross-tile prefix by decoupled look-back ----

template <int kItems, int kWindow, bool kBallot>
__global__ void __launch_bounds__(kThreads, kItems == 8 ? 5 : 4) onesweep_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, uint32_t count,
    const uint32_t* __restrict__ live_count, int drop, int shift, int bits,
    const uint32_t* __restrict__ hist, uint32_t* __restrict__ counter,
    uint32_t* __restrict__ status, uint32_t* __restrict__ error, uint32_t stall_tile) {
    constexpr uint32_t kTileItems = PassTile<kItems>::kTileItems;
    __shared__ PassTile<kItems> t;
    // An earlier pass gave up a wait: its output is not a permutation of the
    // input, so this pass's histogram no longer matches it. Every block leaves.
    if (wait_failed(error)) return;
    if (threadIdx.x == 0) t.slot = atomicAdd(counter, 1u);
    tile_begin(t);
    // Tiles are numbered in the order blocks start, so every earlier tile's
    // block has started and will publish without waiting on this one.
    const uint32_t tile = t.slot;
    const uint64_t tile_begin_item = static_cast<uint64_t>(tile) * kTileItems;
    // Passes after a dropping first pass sort its *live_count survivors; the
    // grid is sized for all items, and blocks past the survivors leave (no
    // block waits on a later tile).
    const uint32_t items = pass_items(count, live_count);
    if (tile_begin_item >= items) return;
    const uint64_t left = items - tile_begin_item;
    const uint32_t n = left < static_cast<uint64_t>(kTileItems) ? static_cast<uint32_t>(left) : kTileItems;
    tile_issue_load(t, keys_in, vals_in, tile_begin_item, n);
    if (!tile_wait_load(t, error)) return;
    uint32_t rank[kItems];
    const uint32_t total = tile_rank<kItems, kBallot>(t, n, drop, shift, bits, rank);

    // look-back across tiles for this thread's digit
    const int b = threadIdx.x;
    uint32_t* my_status = status + static_cast<uint64_t>(tile) * kBins + b;
    const bool publish = tile != stall_tile;  // test hook: a tile that never publishes
    if (tile == 0) {
        if (publish) store_status(my_status, kFlagInclusive | total);
    } else if (publish) {
        store_status(my_status, kFlagAggregate | total);
    }
    const uint32_t earlier =
        tile == 0 ? 0u : look_back<kWindow>(status + b, tile, kBins, error);
    if (tile != 0 && publish) store_status(my_status, kFlagInclusive | ((earlier + total) & kValueMask));
    // global start of each digit: exclusive scan of the pass histogram
    t.global_base[b] = block_exclusive_256(hist[b], t.warp_sums) + earlier;
    tile_scatter(t, n, drop, shift, bits, total, rank, keys_out, vals_out);
}

// ---- reduce-then-scan pass: count, scan across tiles, scatter ----

// Per tile, the digit counts of its items, stored digit-major:
// counts[digit * tiles + tile]. Tiles past the items write zeros.
template <int kItems>
__global__ void __launch_bounds__(kThreads) count_kernel(
    const uint32_t* __restrict__ keys, uint32_t count, const uint32_t* __restrict__ live_count,
    int drop, int shift, int bits, uint32_t tiles, uint32_t* __restrict__ counts,
    const uint32_t* __restrict__ error) {
    constexpr uint32_t kTileItems = kThreads * kItems;
    __shared__ uint32_t bins[kBins];
    if (wait_failed(error)) return;  // the scan and scatter of this pass leave too
    bins[threadIdx.x] = 0;
    __syncthreads();
    const uint32_t mask = (1u << bits) - 1u;
    const uint32_t items = pass_items(count, live_count);
    const uint64_t begin = static_cast<uint64_t>(blockIdx.x) * kTileItems;
    if (begin < items) {
        const uint32_t n = items - begin < kTileItems ? static_cast<uint32_t>(items - begin) : kTileItems;
        const uint32_t* tile = keys + begin;
        auto add = [&](uint32_t key) {
            if (!(drop && key == kDropKey)) atomicAdd(&bins[digit_of(key, shift, mask)], 1u);
        };
        // 16-byte loads: a tile starts at a multiple of kTileItems items of a
        // 16-byte aligned array
        const uint32_t quads = n / 4u;
        for (uint32_t q = threadIdx.x; q < quads; q += kThreads) {
            const uint4 v = reinterpret_cast<const uint4*>(tile)[q];
            add(v.x);
            add(v.y);
            add(v.z);
            add(v.w);
        }
        if (threadIdx.x < n - quads * 4u) add(tile[quads * 4u + threadIdx.x]);
    }
    __syncthreads();
    counts[static_cast<uint64_t>(threadIdx.x) * tiles + blockIdx.x] = bins[threadIdx.x];
}

// One block per digit: that digit's counts across the tiles replaced by their
// exclusive prefix, and the digit's total.
__global__ void __launch_bounds__(kThreads) scan_kernel(uint32_t* __restrict__ counts, uint32_t tiles,
                                                        uint32_t* __restrict__ totals,
                                                        const uint32_t* __restrict__ error) {
    __shared__ uint32_t warp_sums[kWarps];
    if (wait_failed(error)) return;
    uint32_t* row = counts + static_cast<uint64_t>(blockIdx.x) * tiles;
    const uint32_t per = (tiles + kThreads - 1) / kThreads;
    const uint32_t first = threadIdx.x * per;
    const uint32_t last = min(first + per, tiles);
    uint32_t sum = 0;
    for (uint32_t i = first; i < last; ++i) sum += row[i];
    uint32_t run = block_exclusive_256(sum, warp_sums);
    for (uint32_t i = first; i < last; ++i) {
        const uint32_t c = row[i];
        row[i] = run;
        run += c;
    }
    if (threadIdx.x == kThreads - 1) totals[blockIdx.x] = run;
}

// Tile blockIdx.x ranked and scattered to (start of its digit) + (this tile's
// prefix for the digit); the digit starts are the exclusive scan of the 256
// totals, which every block forms. No block waits on another.
template <int kItems, bool kBallot>
__global__ void __launch_bounds__(kThreads, 4) scatter_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, uint32_t count,
    const uint32_t* __restrict__ live_count, int drop, int shift, int bits, uint32_t tiles,
    const uint32_t* __restrict__ prefix, const uint32_t* __restrict__ totals,
    uint32_t* __restrict__ error) {
    constexpr uint32_t kTileItems = PassTile<kItems>::kTileItems;
    __shared__ PassTile<kItems> t;
    if (wait_failed(error)) return;
    const uint32_t items = pass_items(count, live_count);
    const uint32_t tile = blockIdx.x;
    const uint64_t tile_begin_item = static_cast<uint64_t>(tile) * kTileItems;
    if (tile_begin_item >= items) return;
    tile_begin(t);
    const uint64_t left = items - tile_begin_item;
    const uint32_t n = left < static_cast<uint64_t>(kTileItems) ? static_cast<uint32_t>(left) : kTileItems;
    tile_issue_load(t, keys_in, vals_in, tile_begin_item, n);
    // the destinations do not depend on the tile: formed while it lands
    const int b = threadIdx.x;
    t.global_base[b] = block_exclusive_256(totals[b], t.warp_sums) + prefix[static_cast<uint64_t>(b) * tiles + tile];
    if (!tile_wait_load(t, error)) return;
    uint32_t rank[kItems];
    const uint32_t total = tile_rank<kItems, kBallot>(t, n, drop, shift, bits, rank);
    tile_scatter(t, n, drop, shift, bits, total, rank, keys_out, vals_out);
}

}  // namespace

uint64_t sort_scratch_bytes(uint32_t count) {
    const uint64_t tiles = tiles_for(count > 0 ? count : 1);
    // onesweep: histograms, counters, look-back words of every pass
    const uint64_t onesweep = static_cast<uint64_t>(kMaxPasses) * kBins + 64 + kMaxPasses * tiles * kBins;
    // reduce-then-scan: per-digit counts of every 4096-item tile, the totals
    const uint64_t large_tiles = (static_cast<uint64_t>(count) + kThreads * kLargeItems - 1) / (kThreads * kLargeItems);
    const uint64_t split = static_cast<uint64_t>(kBins) * large_tiles + kBins + 64;
    return (onesweep > split ? onesweep : split) * sizeof(uint32_t);
}

namespace {

// Reduce-then-scan passes (count, scan, scatter kernels per pass).
cudaError_t sort_split(uint32_t*& src_k, uint32_t*& src_v, uint32_t*& dst_k, uint32_t*& dst_v,
                       uint32_t count, int begin_bit, int end_bit, void* scratch, cudaStream_t stream,
                       uint32_t* error, const uint32_t* kept, int drop, bool ballot, const uint32_t* bound) {
    const uint32_t tiles =
        static_cast<uint32_t>((static_cast<uint64_t>(count) + kThreads * kLargeItems - 1) / (kThreads * kLargeItems));
    uint32_t* counts = static_cast<uint32_t*>(scratch);
    uint32_t* totals = counts + static_cast<uint64_t>(kBins) * tiles;
    int pass = 0;
    for (int shift = begin_bit; shift < end_bit; shift += kRadixBits, ++pass) {
        const int bits = min(kRadixBits, end_bit - shift);
        const uint32_t* live = pass > 0 && kept != nullptr ? kept : bound;
        const int pass_drop = pass == 0 ? drop : 0;
        count_kernel<kLargeItems><<<tiles, kThreads, 0, stream>>>(src_k, count, live, pass_drop, shift, bits,
                                                                  tiles, counts, error);
        scan_kernel<<<1u << bits, kThreads, 0, stream>>>(counts, tiles, totals, error);
        if (bits < kRadixBits) {
            // digits from 2^bits on hold no item: their totals are zero
            const cudaError_t st = cudaMemsetAsync(totals + (1u << bits), 0,
                                                   (kBins - (1u << bits)) * sizeof(uint32_t), stream);
            if (st != cudaSuccess) return st;
        }
        if (ballot) {
            scatter_kernel<kLargeItems, true><<<tiles, kThreads, 0, stream>>>(
                src_k, src_v, dst_k, dst_v, count, live, pass_drop, shift, bits, tiles, counts, totals, error);
        } else {
            scatter_kernel<kLargeItems, false><<<tiles, kThreads, 0, stream>>>(
                src_k, src_v, dst_k, dst_v, count, live, pass_drop, shift, bits, tiles, counts, totals, error);
        }
        std::swap(src_k, dst_k);
        std::swap(src_v, dst_v);
    }
    return cudaSuccess;
}

// Onesweep passes (histogram of every pass, then one kernel per pass).
cudaError_t sort_onesweep(uint32_t*& src_k, uint32_t*& src_v, uint32_t*& dst_k, uint32_t*& dst_v,
                          uint32_t count, int begin_bit, int end_bit, void* scratch, cudaStream_t stream,
                          uint32_t* error, uint32_t stall_tile, const uint32_t* kept, int drop, bool ballot,
                          const uint32_t* bound) {
    const uint32_t tiles = tiles_for(count);
    const bool large = count >= kLargeTileItems;
    const uint32_t large_tiles =
        static_cast<uint32_t>((static_cast<uint64_t>(count) + kThreads * kLargeItems - 1) /
                              (kThreads * kLargeItems));
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    // status words are laid out for 2048-item tiles, enough for either size
    const SortScratch s = sort_scratch(scratch, tiles, passes);
    cudaError_t st = cudaMemsetAsync(scratch, 0, s.zero_bytes, stream);
    if (st != cudaSuccess) return st;
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    const uint32_t hist_cap = static_cast<uint32_t>(sms) * 8u;
    const uint32_t hist_blocks = tiles < hist_cap ? tiles : hist_cap;
    histogram_kernel<<<hist_blocks, kThreads, 0, stream>>>(src_k, count, begin_bit, end_bit, drop, s.hist,
                                                           bound);
    int pass = 0;
    for (int shift = begin_bit; shift < end_bit; shift += kRadixBits, ++pass) {
        const int bits = min(kRadixBits, end_bit - shift);
        const uint32_t stall = pass == 0 ? stall_tile : kNoStall;
        uint32_t* pass_status = s.status + static_cast<uint64_t>(pass) * tiles * kBins;
        // the first pass of a dropping sort reads every item and drops; the
        // later ones sort the *kept survivors
        const uint32_t* live = pass > 0 && kept != nullptr ? kept : bound;
        const int pass_drop = pass == 0 ? drop : 0;
        if (large && ballot) {
            onesweep_kernel<kLargeItems, kLargeWindow, true><<<large_tiles, kThreads, 0, stream>>>(
                src_k, src_v, dst_k, dst_v, count, live, pass_drop, shift, bits,
                s.hist + pass * kBins, s.counters + pass, pass_status, error, stall);
        } else if (large) {
            onesweep_kernel<kLargeItems, kLargeWindow, false><<<large_tiles, kThreads, 0, stream>>>(
                src_k, src_v, dst_k, dst_v, count, live, pass_drop, shift, bits,
                s.hist + pass * kBins, s.counters + pass, pass_status, error, stall);
        } else {
            onesweep_kernel<kItemsPerThread, kLookBackWindow, false>
                <<<tiles, kThreads, 0, stream>>>(src_k, src_v, dst_k, dst_v, count, live,
                                                 pass_drop, shift, bits, s.hist + pass * kBins,
                                                 s.counters + pass, pass_status, error, stall);
        }
        std::swap(src_k, dst_k);
        std::swap(src_v, dst_v);
    }
    return cudaSuccess;
}

}  // namespace

cudaError_t sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals,
                       uint32_t count, int begin_bit, int end_bit, void* scratch,
                       cudaStream_t stream, uint32_t* error, uint32_t stall_tile,
                       const uint32_t* kept, const uint32_t* bound) {
    if (count == 0 || end_bit <= begin_bit) return cudaSuccess;
    if (kept != nullptr && bound != nullptr) return cudaErrorInvalidValue;
    if (count > kMaxItems || end_bit - begin_bit > kMaxPasses * kRadixBits) {
        return cudaErrorInvalidValue;
    }
    // dropping needs the whole key (the dropped key is all ones) and an even
    // pass count (the survivors end in keys/vals without a copy)
    if (kept != nullptr && (begin_bit != 0 || end_bit != 32)) return cudaErrorInvalidValue;
    const int drop = kept != nullptr ? 1 : 0;
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    const bool ballot = passes == kMaxPasses || count >= kBallotItems;
    uint32_t* src_k = keys;
    uint32_t* src_v = vals;
    uint32_t* dst_k = alt_keys;
    uint32_t* dst_v = alt_vals;
    const cudaError_t st =
        count >= kSplitItems
            ? sort_split(src_k, src_v, dst_k, dst_v, count, begin_bit, end_bit, scratch, stream, error, kept,
                         drop, ballot, bound)
            : sort_onesweep(src_k, src_v, dst_k, dst_v, count, begin_bit, end_bit, scratch, stream, error,
                            stall_tile, kept, drop, ballot, bound);
    if (st != cudaSuccess) return st;
    if (passes & 1) {
        cudaError_t cs = cudaMemcpyAsync(keys, src_k, static_cast<size_t>(count) * sizeof(uint32_t),
                                         cudaMemcpyDeviceToDevice, stream);
        if (cs != cudaSuccess) return cs;
        cs = cudaMemcpyAsync(vals, src_v, static_cast<size_t>(count) * sizeof(uint32_t),
                             cudaMemcpyDeviceToDevice, stream);
        if (cs != cudaSuccess) return cs;
    }
    return cudaGetLastError();
}

}  // namespace sort
}  // namespace hs
