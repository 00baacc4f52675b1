// Onesweep stable LSD radix sort (sort.cuh).
//
// Scratch layout of sort_pairs (zeroed by one memset per sort):
//   hist[kMaxPasses][kBins]        digit counts of every pass
//   tile_counter[kMaxPasses]       dynamic tile numbering per pass
//   status[kMaxPasses][tiles][kBins] look-back words
// Each pass kernel block:
//   1. takes the next tile number (so every earlier tile's block has
//      already started and will publish without waiting on this one) and
//      copies the tile's keys and values into shared memory with two bulk
//      asynchronous copies (the TMA engine; a ragged tail of < 4 items with
//      plain loads), so no thread holds the items in registers while ranking;
//   2. ranks its 2048 items stably: warp w owns the contiguous segment
//      [256w, 256w + 256) and walks it 32 items at a time with
//      __match_any_sync on the digit; per-warp digit counts are prefixed
//      across warps;
//   3. publishes its per-digit counts, looks back for the counts of all
//      earlier tiles, publishes the inclusive sums;
//   4. permutes the tile in shared memory into digit order and writes each
//      digit run to consecutive global positions (coalesced).
// Keeping the tile in shared memory instead of registers lets six blocks
// share an SM, which hides the latency of the look-back.
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
                                                             uint32_t* __restrict__ hist) {
    __shared__ uint32_t bins[kMaxPasses][kBins];
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

template <int kItems, int kWindow, bool kBallot>
__global__ void __launch_bounds__(kThreads, kItems == 8 ? 5 : 4) onesweep_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, uint32_t count,
    const uint32_t* __restrict__ live_count, int drop, int shift, int bits,
    const uint32_t* __restrict__ hist, uint32_t* __restrict__ counter,
    uint32_t* __restrict__ status, uint32_t* __restrict__ error, uint32_t stall_tile) {
    constexpr uint32_t kTileItems = kThreads * kItems;
    constexpr uint32_t kWarpItems = kTileItems / kWarps;  // contiguous items per warp
    // The tile, in input order until step 4 permutes it into digit order.
    __shared__ alignas(16) uint32_t tile_keys[kTileItems];
    __shared__ alignas(16) uint32_t tile_vals[kTileItems];
    __shared__ uint32_t warp_count[kWarps][kBins];
    __shared__ uint32_t digit_start[kBins];   // first local position of each digit
    __shared__ uint32_t global_base[kBins];   // destination of the digit run's first item
    __shared__ uint32_t warp_sums[kWarps];
    __shared__ uint32_t tile_slot;
    __shared__ uint32_t tile_kept;            // items of the tile that are written
    __shared__ alignas(8) uint64_t loaded;    // completes when the bulk copies land

    // An earlier pass gave up a wait: its output is not a permutation of the
    // input, so this pass's histogram no longer matches it. Every block leaves.
    if (wait_failed(error)) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t mask = (1u << bits) - 1u;
    if (threadIdx.x == 0) {
        tile_slot = atomicAdd(counter, 1u);
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(shared_address(&loaded))
                     : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int b = lane; b < kBins; b += 32) warp_count[warp][b] = 0;
    __syncthreads();
    const uint32_t tile = tile_slot;
    const uint64_t tile_begin = static_cast<uint64_t>(tile) * kTileItems;
    // Passes after a dropping first pass sort its *live_count survivors; the
    // grid is sized for all items, and blocks past the survivors leave (no
    // block waits on a later tile).
    const uint32_t items = live_count != nullptr ? *live_count : count;
    if (tile_begin >= items) return;
    const uint64_t left = items - tile_begin;
    const uint32_t n = left < static_cast<uint64_t>(kTileItems) ? static_cast<uint32_t>(left)
                                                                : kTileItems;
    const uint32_t bulk = n & ~3u;  // whole 16-byte groups go through the copy engine

    // 1. load the tile
    if (threadIdx.x == 0) {
        if (bulk != 0u) {
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                         ::"r"(shared_address(&loaded)), "r"(2u * bulk * 4u) : "memory");
            bulk_load(tile_keys, keys_in + tile_begin, bulk * 4u, &loaded);
            bulk_load(tile_vals, vals_in + tile_begin, bulk * 4u, &loaded);
        } else {
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                         ::"r"(shared_address(&loaded)) : "memory");
        }
    }
    if (threadIdx.x < n - bulk) {
        tile_keys[bulk + threadIdx.x] = keys_in[tile_begin + bulk + threadIdx.x];
        tile_vals[bulk + threadIdx.x] = vals_in[tile_begin + bulk + threadIdx.x];
    }
    const bool landed = wait_tile(&loaded);
    if (!__syncthreads_and(landed)) {
        // The copies did not complete within the bound: report, wait once more
        // (bounded) so that no copy is left writing this block's shared memory.
        if (threadIdx.x == 0) {
            if (error != nullptr) atomicOr(error, 1u);
            wait_tile(&loaded);
        }
        return;
    }

    // 2. stable ranking within the tile
    const uint32_t seg = static_cast<uint32_t>(warp) * kWarpItems;
    const uint32_t lt_mask = (1u << lane) - 1u;
    uint32_t rank[kItems];
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = seg + static_cast<uint32_t>(k) * 32u + lane;
        const uint32_t key = i < n ? tile_keys[i] : 0u;
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
        const uint32_t before = dig >= 0 ? warp_count[warp][dig] : 0u;
        __syncwarp();
        rank[k] = before + __popc(peers & lt_mask);
        const int leader = __ffs(peers) - 1;
        if (dig >= 0 && lane == leader) warp_count[warp][dig] = before + __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    // per-digit totals of the tile and the exclusive per-warp prefixes
    const int b = threadIdx.x;  // one digit per thread
    uint32_t total = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const uint32_t c = warp_count[w][b];
        warp_count[w][b] = total;
        total += c;
    }

    // 3. look-back across tiles for this digit
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
    const uint32_t digit_global = block_exclusive_256(hist[b], warp_sums);
    const uint32_t local_start = block_exclusive_256(total, warp_sums);
    digit_start[b] = local_start;
    global_base[b] = digit_global + earlier;
    if (b == kBins - 1) tile_kept = local_start + total;

    // 4. permute the tile into digit order in place (keys, then values), then
    //    write digit runs
    uint32_t item[kItems];
    bool keep[kItems];
    __syncthreads();  // digit_start / global_base
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        const uint32_t i = seg + static_cast<uint32_t>(k) * 32u + lane;
        item[k] = tile_keys[i];
        keep[k] = i < n && !(drop && item[k] == kDropKey);
        if (keep[k]) {
            const uint32_t d = digit_of(item[k], shift, mask);
            rank[k] += digit_start[d] + warp_count[warp][d];  // final position in the tile
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        if (keep[k]) tile_keys[rank[k]] = item[k];
    }
#pragma unroll
    for (int k = 0; k < kItems; ++k) item[k] = tile_vals[seg + static_cast<uint32_t>(k) * 32u + lane];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItems; ++k) {
        if (keep[k]) tile_vals[rank[k]] = item[k];
    }
    __syncthreads();
    const uint32_t written = tile_kept;  // n unless the pass drops items
    for (uint32_t i = threadIdx.x; i < written; i += kThreads) {
        const uint32_t k = tile_keys[i];
        const uint32_t d = digit_of(k, shift, mask);
        const uint32_t dst = global_base[d] + (i - digit_start[d]);
        keys_out[dst] = k;
        vals_out[dst] = tile_vals[i];
    }
}

}  // namespace

uint64_t sort_scratch_bytes(uint32_t count) {
    const uint64_t tiles = tiles_for(count > 0 ? count : 1);
    return (static_cast<uint64_t>(kMaxPasses) * kBins + 64 + kMaxPasses * tiles * kBins) *
           sizeof(uint32_t);
}

cudaError_t sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals,
                       uint32_t count, int begin_bit, int end_bit, void* scratch,
                       cudaStream_t stream, uint32_t* error, uint32_t stall_tile,
                       const uint32_t* kept) {
    if (count == 0 || end_bit <= begin_bit) return cudaSuccess;
    if (count > kMaxItems || end_bit - begin_bit > kMaxPasses * kRadixBits) {
        return cudaErrorInvalidValue;
    }
    // dropping needs the whole key (the dropped key is all ones) and an even
    // pass count (the survivors end in keys/vals without a copy)
    if (kept != nullptr && (begin_bit != 0 || end_bit != 32)) return cudaErrorInvalidValue;
    const int drop = kept != nullptr ? 1 : 0;
    const uint32_t tiles = tiles_for(count);
    const bool large = count >= kLargeTileItems;
    const uint32_t large_tiles =
        static_cast<uint32_t>((static_cast<uint64_t>(count) + kThreads * kLargeItems - 1) /
                              (kThreads * kLargeItems));
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    const bool ballot = passes == kMaxPasses || count >= kBallotItems;
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
    histogram_kernel<<<hist_blocks, kThreads, 0, stream>>>(keys, count, begin_bit, end_bit, drop,
                                                           s.hist);
    uint32_t* src_k = keys;
    uint32_t* src_v = vals;
    uint32_t* dst_k = alt_keys;
    uint32_t* dst_v = alt_vals;
    int pass = 0;
    for (int shift = begin_bit; shift < end_bit; shift += kRadixBits, ++pass) {
        const int bits = min(kRadixBits, end_bit - shift);
        const uint32_t stall = pass == 0 ? stall_tile : kNoStall;
        uint32_t* pass_status = s.status + static_cast<uint64_t>(pass) * tiles * kBins;
        // the first pass of a dropping sort reads every item and drops; the
        // later ones sort the *kept survivors
        const uint32_t* live = pass > 0 ? kept : nullptr;
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
        uint32_t* tk = src_k;
        uint32_t* tv = src_v;
        src_k = dst_k;
        src_v = dst_v;
        dst_k = tk;
        dst_v = tv;
    }
    if (pass & 1) {
        st = cudaMemcpyAsync(keys, src_k, static_cast<size_t>(count) * sizeof(uint32_t),
                             cudaMemcpyDeviceToDevice, stream);
        if (st != cudaSuccess) return st;
        st = cudaMemcpyAsync(vals, src_v, static_cast<size_t>(count) * sizeof(uint32_t),
                             cudaMemcpyDeviceToDevice, stream);
        if (st != cudaSuccess) return st;
    }
    return cudaGetLastError();
}

}  // namespace sort
}  // namespace hs
