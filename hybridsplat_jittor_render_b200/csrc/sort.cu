// Stable LSD radix sort and exclusive scan (see sort.cuh).
//
// Radix pass structure (8-bit digits):
//   1. count:   each 2048-item tile builds a 256-bin digit histogram in shared
//               memory and stores it bin-major: hist[bin * tiles + tile].
//   2. scan:    one block turns hist into exclusive global offsets; bin-major
//               order makes each (bin, tile) offset account for every
//               smaller bin and every earlier tile of the same bin.
//   3. scatter: each warp ranks its contiguous 256-item segment in order,
//               32 items at a time, with __match_any_sync on the digit; per-warp
//               digit counts are prefixed across the 8 warps, so the final
//               position keeps the input order among equal digits (stable).
#include "sort.cuh"

namespace hs {
namespace sort {
namespace {

constexpr int kWarps = kThreads / 32;
constexpr int kWarpItems = kTile / kWarps;  // 256 contiguous items per warp

__device__ __forceinline__ uint32_t digit_of(uint32_t key, int shift) {
    return (key >> shift) & (kBins - 1);
}

__global__ void __launch_bounds__(kThreads) count_kernel(const uint32_t* __restrict__ keys,
                                                         uint32_t count, int shift,
                                                         uint32_t tiles,
                                                         uint32_t* __restrict__ hist) {
    __shared__ uint32_t bins[kBins];
    bins[threadIdx.x] = 0;
    __syncthreads();
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kTile;
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint64_t i = base + static_cast<uint64_t>(k) * kThreads + threadIdx.x;
        if (i < count) atomicAdd(&bins[digit_of(keys[i], shift)], 1u);
    }
    __syncthreads();
    hist[static_cast<uint64_t>(threadIdx.x) * tiles + blockIdx.x] = bins[threadIdx.x];
}

// Single-block exclusive scan of n values in place (n up to a few million).
__global__ void __launch_bounds__(1024) scan_inplace_kernel(uint32_t* __restrict__ data,
                                                            uint64_t n,
                                                            uint32_t* __restrict__ total) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (uint64_t start = 0; start < n; start += 1024ull * 4ull) {
        // Each thread owns 4 consecutive values.
        const uint64_t i0 = start + static_cast<uint64_t>(threadIdx.x) * 4ull;
        uint32_t v[4];
        uint32_t local = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[k] = (i0 + k < n) ? data[i0 + k] : 0u;
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
        if (warp == 0) {
            uint32_t w = warp_sums[lane];
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, w, off);
                if (lane >= off) w += t;
            }
            warp_sums[lane] = w;  // inclusive
        }
        __syncthreads();
        uint32_t run = carry + (warp > 0 ? warp_sums[warp - 1] : 0u) + (incl - local);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (i0 + k < n) data[i0 + k] = run;
            run += v[k];
        }
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_sums[31];
        __syncthreads();
    }
    if (threadIdx.x == 0 && total != nullptr) *total = carry;
}

__global__ void __launch_bounds__(kThreads) scatter_kernel(
    const uint32_t* __restrict__ keys_in, const uint32_t* __restrict__ vals_in,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ vals_out, uint32_t count, int shift,
    uint32_t tiles, const uint32_t* __restrict__ offsets) {
    __shared__ uint32_t warp_count[kWarps][kBins];
    __shared__ uint32_t tile_base[kBins];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int b = lane; b < kBins; b += 32) warp_count[warp][b] = 0;
    tile_base[threadIdx.x] =
        offsets[static_cast<uint64_t>(threadIdx.x) * tiles + blockIdx.x];
    __syncwarp();

    const uint64_t seg = static_cast<uint64_t>(blockIdx.x) * kTile +
                         static_cast<uint64_t>(warp) * kWarpItems;
    const uint32_t lt_mask = (1u << lane) - 1u;
    uint32_t key[kItemsPerThread], val[kItemsPerThread], pos[kItemsPerThread];
    int dig[kItemsPerThread];
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint64_t i = seg + static_cast<uint64_t>(k) * 32 + lane;
        const bool valid = i < count;
        key[k] = valid ? keys_in[i] : 0u;
        val[k] = valid ? vals_in[i] : 0u;
        dig[k] = valid ? static_cast<int>(digit_of(key[k], shift)) : -1;
        const uint32_t peers = __match_any_sync(0xffffffffu, dig[k]);
        const uint32_t before = warp_count[warp][valid ? dig[k] : 0];
        __syncwarp();
        pos[k] = before + __popc(peers & lt_mask);
        const int leader = __ffs(peers) - 1;
        if (valid && lane == leader) warp_count[warp][dig[k]] = before + __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    // Exclusive prefix of the per-warp counts for each digit.
    {
        const int b = threadIdx.x;
        uint32_t run = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const uint32_t c = warp_count[w][b];
            warp_count[w][b] = run;
            run += c;
        }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        if (dig[k] < 0) continue;
        const uint32_t dst = tile_base[dig[k]] + warp_count[warp][dig[k]] + pos[k];
        keys_out[dst] = key[k];
        vals_out[dst] = val[k];
    }
}

// Block reduction for the large scan: per-tile sums of in[gather[i]].
__global__ void __launch_bounds__(kThreads) tile_sum_kernel(const uint32_t* __restrict__ in,
                                                            const uint32_t* __restrict__ gather,
                                                            uint32_t count,
                                                            uint32_t* __restrict__ sums) {
    __shared__ uint32_t warp_sums[kWarps];
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kTile;
    uint32_t s = 0;
#pragma unroll
    for (int k = 0; k < kItemsPerThread; ++k) {
        const uint64_t i = base + static_cast<uint64_t>(k) * kThreads + threadIdx.x;
        if (i < count) s += in[gather != nullptr ? gather[i] : i];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
    if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t t = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) t += warp_sums[w];
        sums[blockIdx.x] = t;
    }
}

// Per-tile exclusive scan plus the tile's global offset.
__global__ void __launch_bounds__(kThreads) tile_scan_kernel(const uint32_t* __restrict__ in,
                                                             const uint32_t* __restrict__ gather,
                                                             uint32_t count,
                                                             const uint32_t* __restrict__ offsets,
                                                             uint32_t* __restrict__ out) {
    __shared__ uint32_t warp_sums[kWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // Blocked arrangement: thread t owns items [t*8, t*8+8) of the tile.
    const uint64_t base = static_cast<uint64_t>(blockIdx.x) * kTile +
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
    uint32_t prefix = offsets[blockIdx.x];
    for (int w = 0; w < warp; ++w) prefix += warp_sums[w];
    uint32_t run = prefix + incl - local;
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
    const uint64_t hist = tiles * kBins;
    return (hist + 64) * sizeof(uint32_t) + scan_scratch_bytes(static_cast<uint32_t>(hist));
}

uint64_t scan_scratch_bytes(uint32_t count) {
    const uint64_t tiles = tiles_for(count > 0 ? count : 1);
    return (tiles + 64) * sizeof(uint32_t);
}

cudaError_t sort_pairs(uint32_t* keys, uint32_t* vals, uint32_t* alt_keys, uint32_t* alt_vals,
                       uint32_t count, int begin_bit, int end_bit, void* scratch,
                       cudaStream_t stream) {
    if (count == 0 || end_bit <= begin_bit) return cudaSuccess;
    const uint32_t tiles = tiles_for(count);
    const uint32_t hist_count = tiles * kBins;
    uint32_t* hist = static_cast<uint32_t*>(scratch);
    void* scan_scratch = hist + hist_count + 64;
    uint32_t* src_k = keys;
    uint32_t* src_v = vals;
    uint32_t* dst_k = alt_keys;
    uint32_t* dst_v = alt_vals;
    int passes = 0;
    for (int shift = begin_bit; shift < end_bit; shift += kRadixBits) {
        count_kernel<<<tiles, kThreads, 0, stream>>>(src_k, count, shift, tiles, hist);
        exclusive_scan(hist, nullptr, hist, nullptr, hist_count, scan_scratch, stream);
        scatter_kernel<<<tiles, kThreads, 0, stream>>>(src_k, src_v, dst_k, dst_v, count, shift,
                                                       tiles, hist);
        uint32_t* tk = src_k;
        uint32_t* tv = src_v;
        src_k = dst_k;
        src_v = dst_v;
        dst_k = tk;
        dst_v = tv;
        ++passes;
    }
    if (passes & 1) {
        cudaMemcpyAsync(keys, src_k, static_cast<size_t>(count) * sizeof(uint32_t),
                        cudaMemcpyDeviceToDevice, stream);
        cudaMemcpyAsync(vals, src_v, static_cast<size_t>(count) * sizeof(uint32_t),
                        cudaMemcpyDeviceToDevice, stream);
    }
    return cudaGetLastError();
}

cudaError_t exclusive_scan(const uint32_t* in, const uint32_t* gather, uint32_t* out,
                           uint32_t* total, uint32_t count, void* scratch,
                           cudaStream_t stream) {
    if (count == 0) {
        if (total != nullptr) return cudaMemsetAsync(total, 0, sizeof(uint32_t), stream);
        return cudaSuccess;
    }
    const uint32_t tiles = tiles_for(count);
    uint32_t* sums = static_cast<uint32_t*>(scratch);
    tile_sum_kernel<<<tiles, kThreads, 0, stream>>>(in, gather, count, sums);
    scan_inplace_kernel<<<1, 1024, 0, stream>>>(sums, tiles, total);
    tile_scan_kernel<<<tiles, kThreads, 0, stream>>>(in, gather, count, sums, out);
    return cudaGetLastError();
}

}  // namespace sort
}  // namespace hs
