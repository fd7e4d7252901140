// sort.cu - device-wide exclusive scan and stable LSD radix sort.
//
// Scan: reduce-then-scan in three launches (block sums, one-block scan of the sums, block scans
// plus offsets). Radix sort: per 8-bit digit a histogram launch (warp-aggregated shared-memory
// counters), a scan of the digit-major [digit][block] count table, and a scatter launch that ranks
// the block's 4096 pairs stably in shared memory (match.any per warp, warp-ordered prefix per digit)
// and writes them out digit run by digit run, so consecutive threads store consecutive addresses.
#include "sort.cuh"

namespace splat {
namespace {

__device__ __forceinline__ uint32_t warp_inclusive_scan(uint32_t v, int lane) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFullMask, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

__device__ __forceinline__ uint32_t warp_sum(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
    return v;
}

// Exclusive scan of one value per thread over the whole block (blockDim.x a multiple of 32,
// at most 1024). s_warp must hold 33 entries. Ends with a barrier so s_warp can be reused.
__device__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_warp, uint32_t& block_total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_warps = blockDim.x >> 5;
    const uint32_t inc = warp_inclusive_scan(v, lane);
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = lane < n_warps ? s_warp[lane] : 0u;
        const uint32_t wi = warp_inclusive_scan(w, lane);
        s_warp[lane] = wi - w;
        if (lane == 31) s_warp[32] = wi;
    }
    __syncthreads();
    const uint32_t res = inc - v + s_warp[warp];
    block_total = s_warp[32];
    __syncthreads();
    return res;
}

__global__ void __launch_bounds__(kScanThreads) k_scan_reduce(const uint32_t* __restrict__ in, long long n,
                                                              uint32_t* __restrict__ partial) {
    __shared__ uint32_t s_warp[32];
    const long long base = static_cast<long long>(blockIdx.x) * kScanTile;
    uint32_t sum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const long long i = base + k * kScanThreads + threadIdx.x;
        if (i < n) sum += in[i];
    }
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t v = s_warp[threadIdx.x];
        v = warp_sum(v);
        if (threadIdx.x == 0) partial[blockIdx.x] = v;
    }
}

// One block: exclusive scan of the per-block sums, in chunks of kScanTile with a running carry.
__global__ void __launch_bounds__(kScanThreads) k_scan_partials(uint32_t* __restrict__ partial, long long nb,
                                                                uint32_t* __restrict__ total) {
    __shared__ uint32_t s_warp[33];
    uint32_t carry = 0;
    for (long long c = 0; c < nb; c += kScanTile) {
        uint32_t v[kScanItems];
        uint32_t tsum = 0;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            const long long i = c + static_cast<long long>(threadIdx.x) * kScanItems + k;
            v[k] = i < nb ? partial[i] : 0u;
            tsum += v[k];
        }
        uint32_t btotal;
        uint32_t run = block_exclusive_scan(tsum, s_warp, btotal) + carry;
#pragma unroll
        for (int k = 0; k < kScanItems; ++k) {
            const long long i = c + static_cast<long long>(threadIdx.x) * kScanItems + k;
            if (i < nb) partial[i] = run;
            run += v[k];
        }
        carry += btotal;
    }
    if (threadIdx.x == 0 && total) *total = carry;
}

__global__ void __launch_bounds__(kScanThreads) k_scan_apply(const uint32_t* in, uint32_t* out, long long n,
                                                             const uint32_t* __restrict__ partial) {
    __shared__ uint32_t s_data[kScanTile];
    __shared__ uint32_t s_warp[33];
    const long long base = static_cast<long long>(blockIdx.x) * kScanTile;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int li = k * kScanThreads + threadIdx.x;
        const long long i = base + li;
        s_data[li] = i < n ? in[i] : 0u;
    }
    __syncthreads();
    uint32_t v[kScanItems];
    uint32_t tsum = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = s_data[threadIdx.x * kScanItems + k];
        tsum += v[k];
    }
    uint32_t btotal;
    uint32_t run = block_exclusive_scan(tsum, s_warp, btotal) + partial[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        s_data[threadIdx.x * kScanItems + k] = run;
        run += v[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const int li = k * kScanThreads + threadIdx.x;
        const long long i = base + li;
        if (i < n) out[i] = s_data[li];
    }
}

template <typename K>
__device__ __forceinline__ uint32_t digit_of(K key, int shift, uint32_t mask) {
    return static_cast<uint32_t>(key >> shift) & mask;
}

// Lanes of the warp whose digit equals this lane's (among the lanes in `valid`): one ballot per digit bit.
__device__ __forceinline__ unsigned digit_peers(uint32_t d, int bits, unsigned valid) {
    unsigned peers = valid;
#pragma unroll
    for (int b = 0; b < kRadixBits; ++b) {
        if (b < bits) {
            const bool set = (d >> b) & 1u;
            const unsigned m = __ballot_sync(kFullMask, set);
            peers &= set ? m : ~m;
        }
    }
    return peers;
}

// Per-warp privatised counters in shared memory (no cross-warp contention), summed at the end.
template <typename K>
__global__ void __launch_bounds__(kSortThreads) k_sort_hist(const K* __restrict__ keys, long long n, int shift,
                                                            uint32_t mask, uint32_t* __restrict__ hist,
                                                            int nblocks) {
    constexpr int kWarps = kSortThreads / 32;
    __shared__ uint32_t s_hist[kWarps][kRadix];
    const int warp = threadIdx.x >> 5;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s_hist[w][threadIdx.x] = 0u;
    __syncthreads();
    const long long base = static_cast<long long>(blockIdx.x) * kSortTile;
#pragma unroll 4
    for (int r = 0; r < kSortRounds; ++r) {
        const long long i = base + r * kSortThreads + threadIdx.x;
        if (i < n) atomicAdd(&s_hist[warp][digit_of(keys[i], shift, mask)], 1u);
    }
    __syncthreads();
    uint32_t total = 0u;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) total += s_hist[w][threadIdx.x];
    hist[static_cast<long long>(threadIdx.x) * nblocks + blockIdx.x] = total;
}

template <typename K>
constexpr size_t scatter_smem_bytes() {
    return kSortTile * sizeof(K) + kSortTile * sizeof(uint32_t) +
           (2 * (kSortThreads / 32) * kRadix + 3 * kRadix) * sizeof(uint32_t);
}

template <typename K>
__global__ void __launch_bounds__(kSortThreads) k_sort_scatter(const K* __restrict__ keys_in,
                                                               const uint32_t* __restrict__ vals_in,
                                                               K* __restrict__ keys_out,
                                                               uint32_t* __restrict__ vals_out, long long n,
                                                               int shift, uint32_t mask,
                                                               const uint32_t* __restrict__ offsets,
                                                               int nblocks) {
    static_assert(kRadix == kSortThreads, "one thread per digit");
    constexpr int kWarps = kSortThreads / 32;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    K* s_keys = reinterpret_cast<K*>(smem_raw);
    uint32_t* s_vals = reinterpret_cast<uint32_t*>(s_keys + kSortTile);
    uint32_t* s_cnt = s_vals + kSortTile;          // [2][kWarps][kRadix]
    uint32_t* s_base = s_cnt + 2 * kWarps * kRadix;  // running count per digit
    uint32_t* s_start = s_base + kRadix;             // first slot of each digit in the sorted tile
    uint32_t* s_goff = s_start + kRadix;             // first global slot of each digit for this block
    __shared__ uint32_t s_warp[33];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bits = __popc(mask);
    s_base[tid] = 0u;
    s_goff[tid] = offsets[static_cast<long long>(tid) * nblocks + blockIdx.x];
#pragma unroll
    for (int w = 0; w < 2 * kWarps; ++w) s_cnt[w * kRadix + tid] = 0u;
    __syncthreads();

    const long long base = static_cast<long long>(blockIdx.x) * kSortTile;
    const int tile_n = static_cast<int>(min(static_cast<long long>(kSortTile), n - base));
    K key[kSortRounds];
    uint32_t val[kSortRounds];
    uint32_t rank[kSortRounds];
#pragma unroll
    for (int r = 0; r < kSortRounds; ++r) {
        uint32_t* cnt = s_cnt + (r & 1) * kWarps * kRadix;
        uint32_t* cnt_prev = s_cnt + ((r + 1) & 1) * kWarps * kRadix;
        const int li = r * kSortThreads + tid;
        const bool ok = li < tile_n;
        uint32_t d = 0u, lane_rank = 0u;
        key[r] = K(0);
        val[r] = 0u;
        const unsigned okm = __ballot_sync(kFullMask, ok);
        if (ok) {
            key[r] = keys_in[base + li];
            val[r] = vals_in[base + li];
            d = digit_of(key[r], shift, mask);
        }
        const unsigned peers = digit_peers(d, bits, okm);
        if (ok) {
            lane_rank = __popc(peers & ((1u << lane) - 1u));
            if (lane_rank == 0u) cnt[warp * kRadix + d] = __popc(peers);
        }
        __syncthreads();
        {   // thread tid owns digit tid: warp-ordered exclusive prefix, then the running count
            uint32_t run = s_base[tid];
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const uint32_t c = cnt[w * kRadix + tid];
                cnt[w * kRadix + tid] = run;
                run += c;
                cnt_prev[w * kRadix + tid] = 0u;  // every read of the previous round's table is done
            }
            s_base[tid] = run;
        }
        __syncthreads();
        rank[r] = ok ? cnt[warp * kRadix + d] + lane_rank : 0u;
    }
    uint32_t btotal;
    s_start[tid] = block_exclusive_scan(s_base[tid], s_warp, btotal);
    __syncthreads();
#pragma unroll
    for (int r = 0; r < kSortRounds; ++r) {
        const int li = r * kSortThreads + tid;
        if (li < tile_n) {
            const uint32_t pos = s_start[digit_of(key[r], shift, mask)] + rank[r];
            s_keys[pos] = key[r];
            s_vals[pos] = val[r];
        }
    }
    __syncthreads();
    for (int li = tid; li < tile_n; li += kSortThreads) {
        const K k = s_keys[li];
        const uint32_t d = digit_of(k, shift, mask);
        const long long g = static_cast<long long>(s_goff[d]) + (li - static_cast<int>(s_start[d]));
        keys_out[g] = k;
        vals_out[g] = s_vals[li];
    }
}

template <typename K>
int configure_scatter() {
    static bool done = false;  // one attribute call per instantiation and process
    if (!done) {
        SPLAT_CUDA(cudaFuncSetAttribute(k_sort_scatter<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(scatter_smem_bytes<K>())));
        done = true;
    }
    return SPLAT_OK;
}

}  // namespace

size_t scan_workspace_bytes(long long n) {
    const long long nb = n > 0 ? div_up(n, kScanTile) : 1;
    return static_cast<size_t>(nb) * sizeof(uint32_t) + 256;
}

int scan_exclusive_u32(const uint32_t* in, uint32_t* out, long long n, uint32_t* total, void* ws,
                       size_t ws_bytes, cudaStream_t stream) {
    if (n <= 0) {
        if (total) SPLAT_CUDA(cudaMemsetAsync(total, 0, sizeof(uint32_t), stream));
        return SPLAT_OK;
    }
    SPLAT_REQUIRE(ws_bytes >= scan_workspace_bytes(n), "scan workspace too small (%zu < %zu)", ws_bytes,
                  scan_workspace_bytes(n));
    const unsigned int nb = div_up(n, kScanTile);
    uint32_t* partial = static_cast<uint32_t*>(ws);
    k_scan_reduce<<<nb, kScanThreads, 0, stream>>>(in, n, partial);
    k_scan_partials<<<1, kScanThreads, 0, stream>>>(partial, nb, total);
    k_scan_apply<<<nb, kScanThreads, 0, stream>>>(in, out, n, partial);
    return check_launch("scan_exclusive_u32");
}

template <typename K>
size_t sort_workspace_bytes(long long n) {
    if (n < 1) n = 1;
    const long long nb = div_up(n, kSortTile);
    Carver c(nullptr, 0);
    c.take<K>(n);
    c.take<uint32_t>(n);
    c.take<uint32_t>(nb * kRadix);
    c.take<unsigned char>(scan_workspace_bytes(nb * kRadix));
    return c.used + 256;
}

template <typename K>
int radix_sort_pairs(const K* keys_in, const uint32_t* vals_in, K* keys_out, uint32_t* vals_out, long long n,
                     int begin_bit, int end_bit, void* ws, size_t ws_bytes, cudaStream_t stream) {
    constexpr int kKeyBits = static_cast<int>(sizeof(K) * 8);
    SPLAT_REQUIRE(0 <= begin_bit && begin_bit <= end_bit && end_bit <= kKeyBits, "bad bit range [%d, %d)",
                  begin_bit, end_bit);
    SPLAT_REQUIRE(n >= 0 && n < (1ll << 31), "sort size %lld out of range", n);
    if (n == 0) return SPLAT_OK;
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    if (passes == 0) {
        SPLAT_CUDA(cudaMemcpyAsync(keys_out, keys_in, n * sizeof(K), cudaMemcpyDeviceToDevice, stream));
        SPLAT_CUDA(cudaMemcpyAsync(vals_out, vals_in, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, stream));
        return SPLAT_OK;
    }
    SPLAT_REQUIRE(ws_bytes >= sort_workspace_bytes<K>(n), "sort workspace too small (%zu < %zu)", ws_bytes,
                  sort_workspace_bytes<K>(n));
    SPLAT_TRY(configure_scatter<K>());
    const int nb = static_cast<int>(div_up(n, kSortTile));
    Carver c(ws, ws_bytes);
    K* alt_keys = c.take<K>(n);
    uint32_t* alt_vals = c.take<uint32_t>(n);
    uint32_t* hist = c.take<uint32_t>(static_cast<size_t>(nb) * kRadix);
    void* scan_ws = c.take<unsigned char>(scan_workspace_bytes(static_cast<long long>(nb) * kRadix));
    const K* src_k = keys_in;
    const uint32_t* src_v = vals_in;
    for (int p = 0; p < passes; ++p) {
        const int shift = begin_bit + p * kRadixBits;
        const int bits = min(kRadixBits, end_bit - shift);
        const uint32_t mask = (1u << bits) - 1u;
        const bool to_out = ((passes - 1 - p) % 2) == 0;
        K* dst_k = to_out ? keys_out : alt_keys;
        uint32_t* dst_v = to_out ? vals_out : alt_vals;
        k_sort_hist<K><<<nb, kSortThreads, 0, stream>>>(src_k, n, shift, mask, hist, nb);
        SPLAT_TRY(scan_exclusive_u32(hist, hist, static_cast<long long>(nb) * kRadix, nullptr, scan_ws,
                                     scan_workspace_bytes(static_cast<long long>(nb) * kRadix), stream));
        k_sort_scatter<K><<<nb, kSortThreads, scatter_smem_bytes<K>(), stream>>>(src_k, src_v, dst_k, dst_v, n,
                                                                                 shift, mask, hist, nb);
        SPLAT_TRY(check_launch("radix_sort_pairs"));
        src_k = dst_k;
        src_v = dst_v;
    }
    return SPLAT_OK;
}

template size_t sort_workspace_bytes<uint32_t>(long long);
template size_t sort_workspace_bytes<unsigned long long>(long long);
template int radix_sort_pairs<uint32_t>(const uint32_t*, const uint32_t*, uint32_t*, uint32_t*, long long, int,
                                        int, void*, size_t, cudaStream_t);
template int radix_sort_pairs<unsigned long long>(const unsigned long long*, const uint32_t*, unsigned long long*,
                                                  uint32_t*, long long, int, int, void*, size_t, cudaStream_t);

}  // namespace splat

// ---------------------------------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------------------------------
extern "C" {

size_t splat_scan_workspace_size(long long n) { return splat::scan_workspace_bytes(n); }

int splat_scan_exclusive_u32(const uint32_t* in, uint32_t* out, long long n, uint32_t* total, void* workspace,
                             size_t workspace_bytes, void* stream) {
    return splat::scan_exclusive_u32(in, out, n, total, workspace, workspace_bytes, splat::as_stream(stream));
}

size_t splat_sort_workspace_size(long long n, int key_bytes) {
    return key_bytes == 8 ? splat::sort_workspace_bytes<unsigned long long>(n)
                          : splat::sort_workspace_bytes<uint32_t>(n);
}

int splat_radix_sort_pairs(const void* keys_in, const uint32_t* vals_in, void* keys_out, uint32_t* vals_out,
                           long long n, int key_bytes, int begin_bit, int end_bit, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (key_bytes == 8)
        return splat::radix_sort_pairs<unsigned long long>(
            static_cast<const unsigned long long*>(keys_in), vals_in, static_cast<unsigned long long*>(keys_out),
            vals_out, n, begin_bit, end_bit, workspace, workspace_bytes, splat::as_stream(stream));
    if (key_bytes == 4)
        return splat::radix_sort_pairs<uint32_t>(static_cast<const uint32_t*>(keys_in), vals_in,
                                                 static_cast<uint32_t*>(keys_out), vals_out, n, begin_bit, end_bit,
                                                 workspace, workspace_bytes, splat::as_stream(stream));
    splat::set_error("key_bytes must be 4 or 8, got %d", key_bytes);
    return SPLAT_ERR_ARG;
}

}  // extern "C"
