// Onesweep stable LSD radix sort and single-pass exclusive scan (sort.cuh).
//
// Scratch layout of sort_pairs (zeroed by one memset per sort):
//   hist[kMaxPasses][kBins]        digit counts of every pass
//   tile_counter[kMaxPasses]       dynamic tile numbering per pass
//   status[kMaxPasses][tiles][kBins] look-back words
// Each pass kernel block:
//   1. takes the next tile number (so every earlier tile's block has
//      already started and will publish without waiting on this one);
//   2. ranks its 2048 items stably: warp w owns the contiguous segment
//      [256w, 256w + 256) and walks it 32 items at a time with
//      __match_any_sync on the digit; per-warp digit counts are prefixed
//      across warps;
//   3. publishes its per-digit counts, looks back for the counts of all
//      earlier tiles, publishes the inclusive sums;
//   4. stages the tile in shared memory in digit order and writes each digit
//      run to consecutive global positions (coalesced).
#include "sort.cuh"

namespace hs {
namespace sort {
namespace {

constexpr int kWarps = kThreads / 32;
constexpr int kWarpItems = kTile / kWarps;  // 256 contiguous items per warp

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

__global__ void __launch_bounds__(kThreads) histogram_kernel(const uint32_t* __restrict__ keys,
                                                             uint32_t count, int begin_bit,
                                                             int end_bit,
                                                             uint32_t* __restrict__ hist) {
    __shared__ uint32_t bins[kMaxPasses][kBins];
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    for (int p = 0; p < passes; ++p) bins[p][threadIdx.x] = 0;
    __syncthreads();
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * kThreads;
    for (uint64_t i = static_cast<uint64_t>(blockIdx.x) * kThreads + threadIdx.x; i < count;
         i += stride) {
        const uint32_t key = keys[i];
        for (int p = 0; p < passes; ++p) {
            const int shift = begin_bit + p * kRadixBits;
            const int bits = min(kRadixBits, end_bit - shift);
            atomicAdd(&bins[p][digit_of(key, shift, (1u << bits) - 1u)], 1u);
        }
    }
    __syncthreads();
    for (int p = 0; p < passes; ++p) {
        const uint32_t v = bins[p][threadIdx.x];
        if (v != 0u) atomicAdd(&hist[p * kBins + threadIdx.x], v);
    }
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

__global__ void __launch_bounds__(kThreads) onesweep_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, uint32_t count, int shift,
    int bits, uint32_t tiles, const uint32_t* __restrict__ hist, uint32_t* __restrict__ counter,
    uint32_t* __restrict__ status, uint32_t* __restrict__ error) {
    __shared__ uint32_t warp_count[kWarps][kBins];
    __shared__ uint32_t digit_start[kBins];   // first local position of each digit
    __shared__ uint32_t global_base[kBins];   // destination of the digit run's first item
    __shared__ uint32_t warp_sums[kWarps];
    __shared__ uint32_t stage_keys[kTile];
    __shared__ uint32_t stage_vals[kTile];
    __shared__ uint32_t tile_slot;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t mask = (1u << bits) - 1u;
    if (threadIdx.x == 0) tile_slot = atomicAdd(counter, 1u);
    for (int b = lane; b < kBins; b += 32) warp_count[warp][b] = 0;
    __syncthreads();
    const uint32_t tile = tile_slot;

    // 2. stable ranking within the tile
    const uint64_t seg = static_cast<uint64_t>(tile) * kTile +
                         static_cast<uint64_t>(warp) * kWarpItems;
    const uint32_t lt_mask = (1u << lane) - 1u;
    uint32_t key[kItemsPerThread], val[kItemsPerThread], rank[kItemsPerThread];
    int dig[kItemsPerThread];
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint64_t i = seg + static_cast<uint64_t>(k) * 32 + lane;
        const bool valid = i < count;
        key[k] = valid ? keys_in[i] : 0u;
        val[k] = valid ? vals_in[i] : 0u;
        dig[k] = valid ? static_cast<int>(digit_of(key[k], shift, mask)) : -1;
    }
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint32_t peers = __match_any_sync(0xffffffffu, dig[k]);
        const uint32_t before = dig[k] >= 0 ? warp_count[warp][dig[k]] : 0u;
        __syncwarp();
        rank[k] = before + __popc(peers & lt_mask);
        const int leader = __ffs(peers) - 1;
        if (dig[k] >= 0 && lane == leader) warp_count[warp][dig[k]] = before + __popc(peers);
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
    if (tile == 0) {
        store_status(my_status, kFlagInclusive | total);
    } else {
        store_status(my_status, kFlagAggregate | total);
    }
    const uint32_t earlier = tile == 0 ? 0u : look_back(status + b, tile, kBins, error);
    if (tile != 0) store_status(my_status, kFlagInclusive | ((earlier + total) & kValueMask));

    // global start of each digit: exclusive scan of the pass histogram
    const uint32_t digit_global = block_exclusive_256(hist[b], warp_sums);
    const uint32_t local_start = block_exclusive_256(total, warp_sums);
    digit_start[b] = local_start;
    global_base[b] = digit_global + earlier;
    __syncthreads();

    // 4. stage in digit order, then write digit runs
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        if (dig[k] < 0) continue;
        const uint32_t pos = digit_start[dig[k]] + warp_count[warp][dig[k]] + rank[k];
        stage_keys[pos] = key[k];
        stage_vals[pos] = val[k];
    }
    __syncthreads();
    const uint64_t tile_begin = static_cast<uint64_t>(tile) * kTile;
    const uint64_t left = count - tile_begin;
    const uint32_t n = left < static_cast<uint64_t>(kTile) ? static_cast<uint32_t>(left) : kTile;
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        const uint32_t k = stage_keys[i];
        const uint32_t d = digit_of(k, shift, mask);
        const uint32_t dst = global_base[d] + (i - digit_start[d]);
        keys_out[dst] = k;
        vals_out[dst] = stage_vals[i];
    }
}

// Single-pass exclusive scan with decoupled look-back; one status word per
// tile follows the counter word in scratch.
__global__ void __launch_bounds__(kThreads) scan_kernel(const uint32_t* in,
                                                        const uint32_t* __restrict__ gather,
                                                        uint32_t* out, uint32_t* total,
                                                        uint32_t count, uint32_t tiles,
                                                        uint32_t* __restrict__ counter,
                                                        uint32_t* __restrict__ status,
                                                        uint32_t* __restrict__ error) {
    __shared__ uint32_t warp_sums[kWarps];
    __shared__ uint32_t tile_slot, tile_prefix;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) tile_slot = atomicAdd(counter, 1u);
    __syncthreads();
    const uint32_t tile = tile_slot;
    // blocked arrangement: thread t owns items [8t, 8t + 8) of the tile
    const uint64_t base = static_cast<uint64_t>(tile) * kTile +
                          static_cast<uint64_t>(threadIdx.x) * kItemsPerThread;
    uint32_t v[kItemsPerThread];
    uint32_t local = 0;
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint64_t i = base + k;
        v[k] = i < count ? in[gather != nullptr ? gather[i] : i] : 0u;
        local += v[k];
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
        for (int w = 0; w < kWarps; ++w) sum += warp_sums[w];
        uint32_t earlier = 0;
        if (tile == 0) {
            store_status(status, kFlagInclusive | (sum & kValueMask));
        } else {
            store_status(status + tile, kFlagAggregate | (sum & kValueMask));
            earlier = look_back(status, tile, 1, error);
            store_status(status + tile, kFlagInclusive | ((earlier + sum) & kValueMask));
        }
        tile_prefix = earlier;
        if (tile == tiles - 1 && total != nullptr) *total = earlier + sum;
    }
    __syncthreads();
    uint32_t run = tile_prefix;
    for (int w = 0; w < warp; ++w) run += warp_sums[w];
    run += incl - local;
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint64_t i = base + k;
        if (i < count) out[i] = run;
        run += v[k];
    }
}

}  // namespace

uint64_t sort_scratch_bytes(uint32_t count) {
    const uint64_t tiles = tiles_for(count > 0 ? count : 1);
    return (static_cast<uint64_t>(kMaxPasses) * kBins + 64 + kMaxPasses * tiles * kBins) *
           sizeof(uint32_t);
}

uint64_t scan_scratch_bytes(uint32_t count) {
    const uint64_t tiles = tiles_for(count > 0 ? count : 1);
    return (tiles + 64) * sizeof(uint32_t);
}

cudaError_t sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals,
                       uint32_t count, int begin_bit, int end_bit, void* scratch,
                       cudaStream_t stream, uint32_t* error) {
    if (count == 0 || end_bit <= begin_bit) return cudaSuccess;
    if (count > kMaxItems || end_bit - begin_bit > kMaxPasses * kRadixBits) {
        return cudaErrorInvalidValue;
    }
    const uint32_t tiles = tiles_for(count);
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    const SortScratch s = sort_scratch(scratch, tiles, passes);
    cudaError_t st = cudaMemsetAsync(scratch, 0, s.zero_bytes, stream);
    if (st != cudaSuccess) return st;
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    const uint32_t hist_cap = static_cast<uint32_t>(sms) * 4u;
    const uint32_t hist_blocks = tiles < hist_cap ? tiles : hist_cap;
    histogram_kernel<<<hist_blocks, kThreads, 0, stream>>>(keys, count, begin_bit, end_bit,
                                                           s.hist);
    uint32_t* src_k = keys;
    uint32_t* src_v = vals;
    uint32_t* dst_k = alt_keys;
    uint32_t* dst_v = alt_vals;
    int pass = 0;
    for (int shift = begin_bit; shift < end_bit; shift += kRadixBits, ++pass) {
        const int bits = min(kRadixBits, end_bit - shift);
        onesweep_kernel<<<tiles, kThreads, 0, stream>>>(
            src_k, src_v, dst_k, dst_v, count, shift, bits, tiles, s.hist + pass * kBins,
            s.counters + pass, s.status + static_cast<uint64_t>(pass) * tiles * kBins, error);
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

cudaError_t exclusive_scan(const uint32_t* in, const uint32_t* gather, uint32_t* out,
                           uint32_t* total, uint32_t count, void* scratch, cudaStream_t stream,
                           uint32_t* error) {
    if (count == 0) {
        if (total != nullptr) return cudaMemsetAsync(total, 0, sizeof(uint32_t), stream);
        return cudaSuccess;
    }
    if (count > kMaxItems) return cudaErrorInvalidValue;
    const uint32_t tiles = tiles_for(count);
    uint32_t* counter = static_cast<uint32_t*>(scratch);
    uint32_t* status = counter + 64;
    cudaError_t st = cudaMemsetAsync(scratch, 0, scan_scratch_bytes(count), stream);
    if (st != cudaSuccess) return st;
    scan_kernel<<<tiles, kThreads, 0, stream>>>(in, gather, out, total, count, tiles, counter,
                                                status, error);
    return cudaGetLastError();
}

}  // namespace sort
}  // namespace hs
