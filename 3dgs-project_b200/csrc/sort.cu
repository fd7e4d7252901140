// sort.cu - device-wide exclusive scan and stable LSD radix sort.
//
// Scan: reduce-then-scan in three launches (block sums, one-block scan of the sums, block scans
// plus offsets). Radix sort: one launch counts the digits of every pass in a single read of the keys,
// one block turns the counts into each digit's first output slot, then one launch per 8-bit digit
// ranks each tile of pairs stably in shared memory (ballot-based digit peers per warp, warp-ordered
// prefix per digit), finds the tile's global offsets by decoupled look-back over the counts the
// earlier tiles publish, and writes the pairs out digit run by digit run, so consecutive threads store
// consecutive addresses.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "sort.cuh"

namespace splat {
namespace {

// Bounded device-side waits that gave up (look-back of the radix sort), per device; read and cleared by
// splat_check_device_waits.
__device__ unsigned int g_wait_timeouts = 0u;


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

// Digit counts of every pass in one read of the keys: per-warp shared counters (dynamic shared memory,
// [passes][warp][digit]), loads batched kHistUnroll deep, then one global atomic per (pass, digit) and block.
constexpr int kHistUnroll = 4;

template <typename K>
__global__ void __launch_bounds__(kSortThreads) k_sort_global_hist(const K* __restrict__ keys, long long n,
                                                                   int begin_bit, int end_bit, int passes,
                                                                   uint32_t* __restrict__ hist,
                                                                   const uint32_t* __restrict__ n_dev) {
    constexpr int kWarps = kSortThreads / 32;
    if (n_dev) n = min(n, static_cast<long long>(*n_dev));  // the count on the device, within the capacity
    extern __shared__ uint32_t s_whist[];
    uint32_t* mine = s_whist + (threadIdx.x >> 5) * kRadix;
    for (int i = threadIdx.x; i < passes * kWarps * kRadix; i += kSortThreads) s_whist[i] = 0u;
    __syncthreads();
    const long long stride = static_cast<long long>(gridDim.x) * kSortThreads;
    auto count = [&](K k) {
        for (int p = 0; p < passes; ++p) {
            const int shift = begin_bit + p * kRadixBits;
            const uint32_t mask = (1u << min(kRadixBits, end_bit - shift)) - 1u;
            atomicAdd(&mine[p * kWarps * kRadix + digit_of(k, shift, mask)], 1u);
        }
    };
    long long i = static_cast<long long>(blockIdx.x) * kSortThreads + threadIdx.x;
    for (; i + (kHistUnroll - 1) * stride < n; i += kHistUnroll * stride) {
        K k[kHistUnroll];
#pragma unroll
        for (int u = 0; u < kHistUnroll; ++u) k[u] = keys[i + u * stride];
#pragma unroll
        for (int u = 0; u < kHistUnroll; ++u) count(k[u]);
    }
    for (; i < n; i += stride) count(keys[i]);
    __syncthreads();
    for (int p = 0; p < passes; ++p) {
        uint32_t total = 0u;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += s_whist[(p * kWarps + w) * kRadix + threadIdx.x];
        if (total) atomicAdd(&hist[p * kRadix + threadIdx.x], total);
    }
}

constexpr size_t global_hist_smem_bytes(int passes) {
    return static_cast<size_t>(passes) * (kSortThreads / 32) * kRadix * sizeof(uint32_t);
}

// hist[p][d] -> first output slot of digit d in pass p (exclusive prefix), one block.
__global__ void __launch_bounds__(kSortThreads) k_sort_digit_base(uint32_t* __restrict__ hist, int passes) {
    __shared__ uint32_t s_warp[33];
    for (int p = 0; p < passes; ++p) {
        uint32_t total;
        const uint32_t v = hist[p * kRadix + threadIdx.x];
        hist[p * kRadix + threadIdx.x] = block_exclusive_scan(v, s_warp, total);
    }
}

// Look-back status words, one per (tile, digit): two flag bits over a 30-bit count.
constexpr uint32_t kAggregateFlag = 1u << 30;  // count of this tile alone
constexpr uint32_t kPrefixFlag = 2u << 30;     // count of this tile and every tile before it
constexpr uint32_t kFlagMask = 3u << 30;
constexpr uint32_t kCountMask = kAggregateFlag - 1u;
// Polls of one digit's look-back before it gives up (about a second with the back-off below; a tile
// normally waits a few microseconds).
constexpr int kLookbackPollLimit = 1 << 20;
// Empty polls a look-back wait makes before it gives up; passed to every scatter launch. Changed only through
// splat_set_lookback_poll_limit (failure-detection tests).
std::atomic<int> g_poll_limit{kLookbackPollLimit};
#ifndef SPLAT_LOOKBACK_WINDOW
#define SPLAT_LOOKBACK_WINDOW 4
#endif
constexpr int kLookbackWindow = SPLAT_LOOKBACK_WINDOW;  // earlier tiles' status words fetched per round trip

__device__ __forceinline__ uint32_t load_status(const uint32_t* p) {
    return *reinterpret_cast<const volatile uint32_t*>(p);
}

__device__ __forceinline__ void store_status(uint32_t* p, uint32_t v) {
    *reinterpret_cast<volatile uint32_t*>(p) = v;
}

template <typename K>
constexpr size_t scatter_smem_bytes() {
    return kSortTile * sizeof(K) + kSortTile * sizeof(uint32_t) +
           (2 * (kSortThreads / 32) * kRadix + 2 * kRadix) * sizeof(uint32_t);
}

// Number of earlier pairs of digit `tid` over all tiles before `tile`: walks back over the status words,
// kLookbackWindow tiles per round trip, summing counts up to and including the first inclusive prefix.
__device__ __forceinline__ uint32_t look_back(const uint32_t* status, long long tile, int tid, int poll_limit,
                                              bool& gave_up) {
    uint32_t excl = 0u;
    long long j = tile - 1;
    int polls = 0;
    while (true) {
        uint32_t st[kLookbackWindow];
#pragma unroll
        for (int q = 0; q < kLookbackWindow; ++q)
            st[q] = j - q >= 0 ? load_status(status + (j - q) * kRadix + tid) : 0u;
        int used = 0;
        bool done = false;
#pragma unroll
        for (int q = 0; q < kLookbackWindow; ++q) {
            // stop at the first tile that has published nothing yet; tile 0 always publishes a prefix,
            // so no entry past it (j - q < 0) is ever consumed
            if (done || used < q || !(st[q] & kFlagMask)) continue;
            excl += st[q] & kCountMask;
            used = q + 1;
            done = (st[q] & kPrefixFlag) != 0u;
        }
        if (done) break;
        j -= used;
        if (used == 0) {
            if (++polls >= poll_limit) {
                atomicAdd(&g_wait_timeouts, 1u);
                gave_up = true;
                break;
            }
            if (polls > 32) __nanosleep(64);
        }
    }
    return excl;
}

// One digit pass in one launch. Tiles are taken in launch order from a ticket counter. Warp w of a tile
// owns the tile's pairs [w * 32 * kSortRounds, (w + 1) * 32 * kSortRounds) and ranks them round by round
// against its own per-digit counters (no block barrier): in a round, each lane ORs its lane bit into its
// digit's match word, so that reading the word back gives the lanes holding the same digit; one block
// barrier later the per-warp counts give each warp's base per digit and the tile's per-digit totals. The
// totals are published, and the number of earlier pairs of each digit is found by looking back over the
// totals of the tiles before (stopping at the first tile that has published an inclusive prefix). A tile
// only waits on tiles that took their ticket earlier, which are running; every wait is bounded, and on
// timeout the wait counter is raised and the tile counts the earlier tiles' digits from the keys themselves (slow,
// exact) instead of hanging.
// Pairs are then placed in digit order in shared memory and written out digit run by digit run.
// kGather: the last pass also writes gather_out[i] = gather_table[value] for every output slot i.
template <typename K, bool kGather>
__global__ void __launch_bounds__(kSortThreads, kSortMinBlocks) k_sort_scatter(const K* __restrict__ keys_in,
                                                               const uint32_t* __restrict__ vals_in,
                                                               K* __restrict__ keys_out,
                                                               uint32_t* __restrict__ vals_out, long long n,
                                                               int shift, uint32_t mask,
                                                               const uint32_t* __restrict__ digit_base,
                                                               uint32_t* __restrict__ status,
                                                               uint32_t* __restrict__ ticket,
                                                               const uint32_t* __restrict__ gather_table,
                                                               uint32_t* __restrict__ gather_out, int poll_limit,
                                                               const uint32_t* __restrict__ n_dev) {
    static_assert(kRadix == kSortThreads, "one thread per digit");
    constexpr int kWarps = kSortThreads / 32;
    constexpr int kWarpItems = 32 * kSortRounds;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    K* s_keys = reinterpret_cast<K*>(smem_raw);
    uint32_t* s_vals = reinterpret_cast<uint32_t*>(s_keys + kSortTile);
    uint32_t* s_cnt = s_vals + kSortTile;          // [kWarps][kRadix]: running counts, then warp bases
    uint32_t* s_match = s_cnt + kWarps * kRadix;   // [kWarps][kRadix]: lanes of the round holding each digit
    uint32_t* s_start = s_match + kWarps * kRadix; // first slot of each digit in the sorted tile
    uint32_t* s_goff = s_start + kRadix;           // first global slot of each digit for this tile
    __shared__ uint32_t s_warp[33];
    __shared__ uint32_t s_tile;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_tile = atomicAdd(ticket, 1u);
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        s_cnt[w * kRadix + tid] = 0u;
        s_match[w * kRadix + tid] = 0u;
    }
    __syncthreads();
    const long long tile = s_tile;
    const long long base = tile * kSortTile;
    if (n_dev) n = min(n, static_cast<long long>(*n_dev));  // the count on the device, within the capacity
    if (base >= n) return;  // a tile past the pairs on the device: no later tile looks back at it
    const int tile_n = static_cast<int>(min(static_cast<long long>(kSortTile), n - base));
    const int wbase = warp * kWarpItems;

    K key[kSortRounds];
    uint32_t val[kSortRounds];
    uint32_t rank[kSortRounds];
#pragma unroll
    for (int r = 0; r < kSortRounds; ++r) {  // every load in flight before the ranking starts
        const int li = wbase + r * 32 + lane;
        key[r] = li < tile_n ? keys_in[base + li] : K(0);
        val[r] = li < tile_n ? vals_in[base + li] : 0u;
    }
    uint32_t* cnt = s_cnt + warp * kRadix;
    uint32_t* match = s_match + warp * kRadix;
    const unsigned lanes_below = (1u << lane) - 1u;
#pragma unroll
    for (int r = 0; r < kSortRounds; ++r) {
        const bool ok = wbase + r * 32 + lane < tile_n;
        const uint32_t d = digit_of(key[r], shift, mask);
        if (ok) atomicOr(&match[d], 1u << lane);
        __syncwarp();
        const unsigned peers = ok ? match[d] : 0u;  // lanes of this round with digit d (this lane included)
        const uint32_t below = __popc(peers & lanes_below);
        const uint32_t prior = ok ? cnt[d] : 0u;
        __syncwarp();
        if (ok && below == 0u) {  // the lowest lane of the group advances the counter and clears the word
            cnt[d] = prior + __popc(peers);
            match[d] = 0u;
        }
        __syncwarp();
        rank[r] = prior + below;
    }
    __syncthreads();
    uint32_t count = 0u;  // thread tid owns digit tid: per-warp counts -> warp bases, tile total
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const uint32_t c = s_cnt[w * kRadix + tid];
        s_cnt[w * kRadix + tid] = count;
        count += c;
    }
    uint32_t* mine = status + tile * kRadix + tid;
    store_status(mine, (tile == 0 ? kPrefixFlag : kAggregateFlag) | count);  // before anything else of the tile
    uint32_t btotal;
    s_start[tid] = block_exclusive_scan(count, s_warp, btotal);  // its barriers publish s_cnt too
    __syncthreads();
    // The tile's pairs in digit order in shared memory first, so that the registers holding them are free during
    // the look-back (its window of status words in flight).
#pragma unroll
    for (int r = 0; r < kSortRounds; ++r) {
        if (wbase + r * 32 + lane < tile_n) {
            const uint32_t d = digit_of(key[r], shift, mask);
            const uint32_t pos = s_start[d] + s_cnt[warp * kRadix + d] + rank[r];
            s_keys[pos] = key[r];
            s_vals[pos] = val[r];
        }
    }
    uint32_t excl = 0u;
    if (tile != 0) {
        bool gave_up = false;
        excl = look_back(status, tile, tid, poll_limit, gave_up);
        if (__syncthreads_or(gave_up)) {
            // A wait gave up (it is counted and reported). The earlier tiles' digit counts are taken from the pass's
            // input itself instead, so the offsets, and the sort, stay exact: the block counts the digits of every
            // key before this tile (in the match words, unused after the ranking).
            s_match[tid] = 0u;
            __syncthreads();
            for (long long i = tid; i < base; i += kSortThreads) atomicAdd(&s_match[digit_of(keys_in[i], shift, mask)], 1u);
            __syncthreads();
            excl = s_match[tid];
        }
        store_status(mine, kPrefixFlag | (excl + count));
    }
    s_goff[tid] = digit_base[tid] + excl;
    __syncthreads();
    for (int li = tid; li < tile_n; li += kSortThreads) {
        const K k = s_keys[li];
        const uint32_t d = digit_of(k, shift, mask);
        const long long g = static_cast<long long>(s_goff[d]) + (li - static_cast<int>(s_start[d]));
        keys_out[g] = k;
        const uint32_t v = s_vals[li];
        vals_out[g] = v;
        if (kGather) gather_out[g] = gather_table[v];
    }
}

template <typename K>
int configure_scatter() {
    static bool done = false;  // one attribute call per instantiation and process
    if (!done) {
        SPLAT_CUDA(cudaFuncSetAttribute(k_sort_scatter<K, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(scatter_smem_bytes<K>())));
        SPLAT_CUDA(cudaFuncSetAttribute(k_sort_scatter<K, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(scatter_smem_bytes<K>())));
        SPLAT_CUDA(cudaFuncSetAttribute(k_sort_global_hist<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(global_hist_smem_bytes(kMaxPasses))));
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
    note_launch();
    k_scan_partials<<<1, kScanThreads, 0, stream>>>(partial, nb, total);
    note_launch();
    k_scan_apply<<<nb, kScanThreads, 0, stream>>>(in, out, n, partial);
    note_launch();
    return check_launch("scan_exclusive_u32");
}

// Workspace layout: alternate keys / values, then one zeroed block (digit counts of every pass, one tile
// ticket per pass, look-back status words of every pass and tile).
template <typename K>
size_t sort_workspace_bytes(long long n) {
    if (n < 1) n = 1;
    const long long nb = div_up(n, kSortTile);
    Carver c(nullptr, 0);
    c.take<K>(n);
    c.take<uint32_t>(n);
    c.take<uint32_t>(kMaxPasses * kRadix + kMaxPasses);
    c.take<uint32_t>(static_cast<size_t>(sizeof(K)) * nb * kRadix);
    return c.used + 256;
}

template <typename K>
int radix_sort_pairs(const K* keys_in, const uint32_t* vals_in, K* keys_out, uint32_t* vals_out, long long n,
                     int begin_bit, int end_bit, void* ws, size_t ws_bytes, cudaStream_t stream,
                     const uint32_t* gather_table, uint32_t* gather_out, const uint32_t* n_dev) {
    constexpr int kKeyBits = static_cast<int>(sizeof(K) * 8);
    SPLAT_REQUIRE(0 <= begin_bit && begin_bit <= end_bit && end_bit <= kKeyBits, "bad bit range [%d, %d)",
                  begin_bit, end_bit);
    SPLAT_REQUIRE(n >= 0 && n <= static_cast<long long>(kCountMask), "sort size %lld out of range (max %u)", n,
                  kCountMask);
    if (n == 0) return SPLAT_OK;
    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    SPLAT_REQUIRE(!gather_out || (gather_table && passes > 0), "radix_sort_pairs: a gather needs a table and a pass");
    if (passes == 0) {
        SPLAT_CUDA(cudaMemcpyAsync(keys_out, keys_in, n * sizeof(K), cudaMemcpyDeviceToDevice, stream));
        SPLAT_CUDA(cudaMemcpyAsync(vals_out, vals_in, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, stream));
        return SPLAT_OK;
    }
    SPLAT_REQUIRE(ws_bytes >= sort_workspace_bytes<K>(n), "sort workspace too small (%zu < %zu)", ws_bytes,
                  sort_workspace_bytes<K>(n));
    SPLAT_TRY(configure_scatter<K>());
    const long long nb = div_up(n, kSortTile);
    Carver c(ws, ws_bytes);
    K* alt_keys = c.take<K>(n);
    uint32_t* alt_vals = c.take<uint32_t>(n);
    uint32_t* hist = c.take<uint32_t>(kMaxPasses * kRadix + kMaxPasses);
    uint32_t* tickets = hist + kMaxPasses * kRadix;
    uint32_t* status = c.take<uint32_t>(static_cast<size_t>(sizeof(K)) * nb * kRadix);
    // hist, tickets and status are contiguous: one memset clears what this sort uses of them.
    const size_t zero_bytes = reinterpret_cast<unsigned char*>(status + static_cast<size_t>(passes) * nb * kRadix) -
                              reinterpret_cast<unsigned char*>(hist);
    SPLAT_CUDA(cudaMemsetAsync(hist, 0, zero_bytes, stream));
    const long long hist_blocks = std::min<long long>(div_up(n, kSortThreads * 8), 4ll * sm_count());
    k_sort_global_hist<K><<<static_cast<unsigned>(hist_blocks), kSortThreads, global_hist_smem_bytes(passes),
                            stream>>>(keys_in, n, begin_bit, end_bit, passes, hist, n_dev);
    note_launch();
    k_sort_digit_base<<<1, kSortThreads, 0, stream>>>(hist, passes);
    note_launch();
    const K* src_k = keys_in;
    const uint32_t* src_v = vals_in;
    for (int p = 0; p < passes; ++p) {
        const int shift = begin_bit + p * kRadixBits;
        const int bits = min(kRadixBits, end_bit - shift);
        const uint32_t mask = (1u << bits) - 1u;
        const bool to_out = ((passes - 1 - p) % 2) == 0;
        K* dst_k = to_out ? keys_out : alt_keys;
        uint32_t* dst_v = to_out ? vals_out : alt_vals;
        const bool gather = gather_out && p == passes - 1;
        auto kernel = gather ? k_sort_scatter<K, true> : k_sort_scatter<K, false>;
        kernel<<<static_cast<unsigned>(nb), kSortThreads, scatter_smem_bytes<K>(), stream>>>(
            src_k, src_v, dst_k, dst_v, n, shift, mask, hist + p * kRadix,
            status + static_cast<size_t>(p) * nb * kRadix, tickets + p, gather_table, gather_out,
            g_poll_limit.load(std::memory_order_relaxed), n_dev);
        note_launch();
        SPLAT_TRY(check_launch("radix_sort_pairs"));
        src_k = dst_k;
        src_v = dst_v;
    }
    return SPLAT_OK;
}

// Moves the wait counter into *dst (device memory) in stream order and clears it.
__global__ void k_take_wait_timeouts(uint32_t* dst) {
    *dst = g_wait_timeouts;
    g_wait_timeouts = 0u;
}

int take_wait_timeouts(unsigned int* count) {
    unsigned int h = 0u;
    SPLAT_CUDA(cudaMemcpyFromSymbol(&h, g_wait_timeouts, sizeof(h)));
    if (h) {
        const unsigned int zero = 0u;
        SPLAT_CUDA(cudaMemcpyToSymbol(g_wait_timeouts, &zero, sizeof(zero)));
    }
    *count = h;
    return SPLAT_OK;
}

// ---- exclusive scan without a workspace: the block sums live in a fixed device array ----

// 2^28 values -> 65,536 block sums of 4096 values: 256 KiB of device memory per device.
constexpr long long kNoAllocScanMaxN = SPLAT_SCAN_NOALLOC_MAX_N;
constexpr long long kNoAllocScanPartials = kNoAllocScanMaxN / kScanTile;
static_assert(kNoAllocScanMaxN % kScanTile == 0, "whole scan blocks");
static __device__ __align__(256) uint32_t g_noalloc_scan_partials[kNoAllocScanPartials];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
uint32_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scan_partials on the current device, looked up on the first call per device.
int noalloc_scan_partials(uint32_t** out) {
    int dev = -1;
    SPLAT_CUDA(cudaGetDevice(&dev));
    SPLAT_REQUIRE(dev >= 0 && dev < kNoAllocMaxDevices, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        SPLAT_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scan_partials));
        g_noalloc_ptr[dev] = static_cast<uint32_t*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return SPLAT_OK;
}

// The array's address is the current device's, so the buffers must be device memory of that device (or managed
// memory): anything else would have the kernels mix this device's scratch with another device's data.
int noalloc_check_pointer(const void* p, const char* name) {
    if (p == nullptr) return SPLAT_OK;
    int dev = -1;
    SPLAT_CUDA(cudaGetDevice(&dev));
    cudaPointerAttributes a{};
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("splat_scan_exclusive_u32_noalloc: %s is not a CUDA pointer (%s)", name, cudaGetErrorString(e));
        return SPLAT_ERR_ARG;
    }
    const bool ok = a.type == cudaMemoryTypeManaged || (a.type == cudaMemoryTypeDevice && a.device == dev);
    SPLAT_REQUIRE(ok, "splat_scan_exclusive_u32_noalloc: %s must be device memory of the current device %d "
                      "(memory type %d on device %d)", name, dev, static_cast<int>(a.type), a.device);
    return SPLAT_OK;
}

}  // namespace

int scan_exclusive_u32_noalloc(const uint32_t* in, uint32_t* out, long long n, uint32_t* total,
                               cudaStream_t stream) {
    if (n > kNoAllocScanMaxN) {
        set_error("splat_scan_exclusive_u32_noalloc: n = %lld exceeds its maximum of %lld values (its fixed "
                  "scratch holds %lld block sums); use splat_scan_exclusive_u32 with a workspace",
                  n, kNoAllocScanMaxN, kNoAllocScanPartials);
        return SPLAT_ERR_OVERFLOW;
    }
    if (n <= 0) {
        if (total) SPLAT_CUDA(cudaMemsetAsync(total, 0, sizeof(uint32_t), stream));
        return SPLAT_OK;
    }
    SPLAT_TRY(noalloc_check_pointer(in, "in"));
    SPLAT_TRY(noalloc_check_pointer(out, "out"));
    SPLAT_TRY(noalloc_check_pointer(total, "total"));
    uint32_t* partial = nullptr;
    SPLAT_TRY(noalloc_scan_partials(&partial));
    const unsigned int nb = div_up(n, kScanTile);  // <= kNoAllocScanPartials
    k_scan_reduce<<<nb, kScanThreads, 0, stream>>>(in, n, partial);
    note_launch();
    k_scan_partials<<<1, kScanThreads, 0, stream>>>(partial, nb, total);
    note_launch();
    k_scan_apply<<<nb, kScanThreads, 0, stream>>>(in, out, n, partial);
    note_launch();
    return check_launch("scan_exclusive_u32_noalloc");
}

template size_t sort_workspace_bytes<uint32_t>(long long);
template size_t sort_workspace_bytes<unsigned long long>(long long);
template int radix_sort_pairs<uint32_t>(const uint32_t*, const uint32_t*, uint32_t*, uint32_t*, long long, int,
                                        int, void*, size_t, cudaStream_t, const uint32_t*, uint32_t*,
                                        const uint32_t*);
template int radix_sort_pairs<unsigned long long>(const unsigned long long*, const uint32_t*, unsigned long long*,
                                                  uint32_t*, long long, int, int, void*, size_t, cudaStream_t,
                                                  const uint32_t*, uint32_t*, const uint32_t*);

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

int splat_set_lookback_poll_limit(int polls) {
    if (polls < 1) {
        splat::set_error("splat_set_lookback_poll_limit: %d polls (at least 1)", polls);
        return -1;
    }
    return splat::g_poll_limit.exchange(polls);
}

int splat_scan_exclusive_u32_noalloc(const uint32_t* in, uint32_t* out, long long n, uint32_t* total, void* stream) {
    return splat::scan_exclusive_u32_noalloc(in, out, n, total, splat::as_stream(stream));
}

size_t splat_sort_workspace_size(long long n, int key_bytes) {
    return key_bytes == 8 ? splat::sort_workspace_bytes<unsigned long long>(n)
                          : splat::sort_workspace_bytes<uint32_t>(n);
}

int splat_take_device_waits_async(uint32_t* dst, void* stream) {
    SPLAT_REQUIRE(dst != nullptr, "splat_take_device_waits_async: dst is NULL");
    splat::k_take_wait_timeouts<<<1, 1, 0, splat::as_stream(stream)>>>(dst);
    splat::note_launch();
    return splat::check_launch("splat_take_device_waits_async");
}

int splat_check_device_waits(void) {
    unsigned int n = 0u;
    SPLAT_TRY(splat::take_wait_timeouts(&n));
    if (n) {
        splat::set_error("%u bounded device-side wait(s) gave up (radix sort look-back; their tiles recounted "
                         "their offsets from the keys, so the sorts are exact, but the device stalled that long)",
                         n);
        return SPLAT_ERR_TIMEOUT;
    }
    return SPLAT_OK;
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
