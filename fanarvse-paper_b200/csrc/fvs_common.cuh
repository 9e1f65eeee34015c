// Shared device helpers of libfanar_b200 (sm_100a): order-preserving keys, block-wide radix select, bitonic sort.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/fanar_b200.h"

#define FVS_CHECK_ARG(cond)            \
    do {                               \
        if (!(cond)) return FVS_EINVAL; \
    } while (0)

static inline int fvs_launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? FVS_OK : (int)e;
}

// Number of SMs of the current device (looked up once per device).
inline int fvs_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    static std::mutex mu;
    static std::map<int, int> cache;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(dev);
    if (it != cache.end()) return it->second;
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
    return n;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device); later calls (including calls made while a
// stream is being captured into a CUDA graph) only read the cache.
inline cudaError_t fvs_ensure_smem(const void* func, size_t bytes) {
    if (bytes <= 48 * 1024) return cudaSuccess;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, size_t> done;
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find({func, dev});
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done[{func, dev}] = bytes;
    return e;
}

namespace fvs {

// tiles of one cell part in the cell-major scans' work lists (entries `cell | part << 16`)
constexpr int CELL_PART_TILES = FVS_CELL_PART_TILES;

constexpr float kNeg = -1e30f;  // the reference's "empty" estimate (`throughput/enginei8.py:48,57`)

// float -> uint32 with the same order (larger float, larger key); NaN is not expected on this path.
__device__ __forceinline__ uint32_t f2o(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float o2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

// atomic max of a float in global memory holding a valid (non-NaN) float: non-negative floats order as signed ints,
// negative ones in reverse as unsigned ints
__device__ __forceinline__ void atomic_max_float(float* addr, float v) {
    if (v >= 0.f)
        atomicMax(reinterpret_cast<int*>(addr), __float_as_int(v));
    else
        atomicMin(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

__device__ __forceinline__ int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// Shared scratch of the block radix select: 256 histogram bins + the running (prefix, rank).
struct SelectScratch {
    unsigned hist[256];
    unsigned long long prefix;
    int rem;
};

// r-th largest (1-based) of the nonzero 32-bit keys held in registers, NK per thread (0 = no key; at least r nonzero
// keys over the block).  The bits above the highest bit in which the largest and the smallest key differ are common to
// all keys and taken as found; the rest are found MSB first, up to 8 bits per pass, from a shared-memory histogram of
// the keys that still match the found prefix.  All threads call it and get the key; *above = #{keys > result} and
// *equal = #{keys == result} (*equal = n when every key is the same, n unknown here: reported as INT_MAX).
struct RegSelectScratch {
    unsigned hist[256];
    uint32_t mx[32], mn[32];
    uint32_t prefix;
    int rem, eq;
};
template <int NK>
__device__ __forceinline__ uint32_t block_rth_largest_reg(const uint32_t (&k)[NK], int r, RegSelectScratch& s,
                                                          int* above, int* equal) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    uint32_t mx = 0u, mn = 0xffffffffu;
#pragma unroll
    for (int i = 0; i < NK; i++) {
        mx = max(mx, k[i]);
        if (k[i] != 0u) mn = min(mn, k[i]);
    }
    mx = __reduce_max_sync(0xffffffffu, mx);
    mn = __reduce_min_sync(0xffffffffu, mn);
    if (lane == 0) {
        s.mx[warp] = mx;
        s.mn[warp] = mn;
    }
    __syncthreads();
    mx = __reduce_max_sync(0xffffffffu, lane < nw ? s.mx[lane] : 0u);
    mn = __reduce_min_sync(0xffffffffu, lane < nw ? s.mn[lane] : 0xffffffffu);
    const uint32_t diff = mx ^ mn;
    int shift = 32 - __clz(diff);  // bits [shift, 32) are common to every key
    if (shift == 0) {
        *above = 0;
        *equal = 0x7fffffff;
        return mx;
    }
    uint32_t prefix = shift == 32 ? 0u : (mx >> shift) << shift;
    int rem = r, eq = 0;
    while (shift > 0) {
        const int lo = shift > 8 ? shift - 8 : 0;
        const uint32_t dmask = (1u << (shift - lo)) - 1u;
        for (int i = tid; i < 256; i += blockDim.x) s.hist[i] = 0u;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < NK; i++) {
            const uint32_t key = k[i];
            if (key != 0u && (shift == 32 || (key >> shift) == (prefix >> shift)))
                atomicAdd(&s.hist[(key >> lo) & dmask], 1u);
        }
        __syncthreads();
        if (warp == 0) {
            // lane l owns bins 255-8l .. 248-8l (descending)
            unsigned c[8], sum = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                c[i] = s.hist[255 - 8 * lane - i];
                sum += c[i];
            }
            unsigned incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const unsigned ball = __ballot_sync(0xffffffffu, incl >= (unsigned)rem);
            const int L = __ffs(ball) - 1;  // always found: the keys matching the prefix number >= rem
            if (lane == L) {
                unsigned before = incl - sum;
                int digit = 0;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    if (before + c[i] >= (unsigned)rem) {
                        digit = 255 - 8 * lane - i;
                        s.eq = (int)c[i];
                        break;
                    }
                    before += c[i];
                }
                s.rem = rem - (int)before;
                s.prefix = prefix | ((uint32_t)digit << lo);
            }
        }
        __syncthreads();
        prefix = s.prefix;
        rem = s.rem;
        eq = s.eq;
        shift = lo;
    }
    *above = r - rem;
    *equal = eq;
    return prefix;
}

// r-th largest (1-based, 1 <= r <= n) of n keys of KBITS bits (32 or 64) produced by key(i); MSB-first radix select,
// 8 bits per pass.  Histogram updates are aggregated per warp (lanes with the same digit add once), since the leading
// digits of scores concentrate in one or two bins.  All threads of the block must call it; every thread gets the key.
template <int KBITS, typename KeyT, typename KeyFn>
__device__ KeyT block_select_rth_largest(KeyFn key, int n, int r, SelectScratch& s) {
    const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31;
    if (tid == 0) {
        s.prefix = 0ull;
        s.rem = r;
    }
    __syncthreads();
#pragma unroll 1
    for (int shift = KBITS - 8; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += nt) s.hist[i] = 0;
        __syncthreads();
        const unsigned long long pre = s.prefix;
        const unsigned long long hmask = (shift + 8 >= 64) ? 0ull : (~0ull << (shift + 8));
        for (int b = tid - lane; b < n; b += nt) {  // whole warps iterate together
            const int i = b + lane;
            bool take = false;
            unsigned digit = 0;
            if (i < n) {
                const unsigned long long k = (unsigned long long)key(i);
                take = (k & hmask) == (pre & hmask);
                digit = (unsigned)(k >> shift) & 255u;
            }
            const unsigned act = __ballot_sync(0xffffffffu, take);
            if (take) {
                const unsigned peers = __match_any_sync(act, digit);
                if ((peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&s.hist[digit], (unsigned)__popc(peers));
            }
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns bins 255-8l .. 248-8l (descending)
            unsigned c[8], sum = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                c[i] = s.hist[255 - 8 * lane - i];
                sum += c[i];
            }
            unsigned incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const int rem = s.rem;
            unsigned ball = __ballot_sync(0xffffffffu, incl >= (unsigned)rem);
            int L = __ffs(ball) - 1;  // always found: the candidates (keys matching the prefix) number >= rem
            if (lane == L) {
                unsigned above = incl - sum;
                int digit = 0;
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    if (above + c[i] >= (unsigned)rem) {
                        digit = 255 - 8 * lane - i;
                        break;
                    }
                    above += c[i];
                }
                s.rem = rem - (int)above;
                s.prefix = pre | ((unsigned long long)digit << shift);
            }
        }
        __syncthreads();
    }
    KeyT res = (KeyT)s.prefix;
    __syncthreads();  // every thread has read the result before the scratch is reused
    return res;
}

// r-th largest (1-based, 1 <= r <= n) of n keys produced by key(i), by ONE warp (all 32 lanes call it); hist is 256
// words of this warp's own shared memory.  Same algorithm as block_select_rth_largest without block barriers.
template <int KBITS, typename KeyT, typename KeyFn>
__device__ KeyT warp_select_rth_largest(KeyFn key, int n, int r, unsigned* hist) {
    const int lane = threadIdx.x & 31;
    unsigned long long prefix = 0ull;
    int rem = r;
#pragma unroll 1
    for (int shift = KBITS - 8; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0;
        __syncwarp();
        const unsigned long long hmask = (shift + 8 >= 64) ? 0ull : (~0ull << (shift + 8));
        for (int b = 0; b < n; b += 32) {
            const int i = b + lane;
            bool take = false;
            unsigned digit = 0;
            if (i < n) {
                const unsigned long long k = (unsigned long long)key(i);
                take = (k & hmask) == (prefix & hmask);
                digit = (unsigned)(k >> shift) & 255u;
            }
            const unsigned act = __ballot_sync(0xffffffffu, take);
            if (take) {
                const unsigned peers = __match_any_sync(act, digit);
                if ((peers & ((1u << lane) - 1u)) == 0u) atomicAdd(&hist[digit], (unsigned)__popc(peers));
            }
        }
        __syncwarp();
        unsigned c[8], sum = 0;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            c[i] = hist[255 - 8 * lane - i];
            sum += c[i];
        }
        unsigned incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        const unsigned ball = __ballot_sync(0xffffffffu, incl >= (unsigned)rem);
        const int L = __ffs(ball) - 1;
        int digit = 0, nrem = rem;
        if (lane == L) {
            unsigned above = incl - sum;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (above + c[i] >= (unsigned)rem) {
                    digit = 255 - 8 * lane - i;
                    break;
                }
                above += c[i];
            }
            nrem = rem - (int)above;
        }
        digit = __shfl_sync(0xffffffffu, digit, L);
        rem = __shfl_sync(0xffffffffu, nrem, L);
        prefix |= (unsigned long long)digit << shift;
        __syncwarp();
    }
    return (KeyT)prefix;
}

// In-place descending bitonic sort of n (a power of two) 64-bit keys in shared memory by one warp.
__device__ __forceinline__ void warp_bitonic_desc(unsigned long long* a, int n) {
    const int lane = threadIdx.x & 31;
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long x = a[i], y = a[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncwarp();
        }
    }
}

// Descending bitonic sort of 32 * PER keys held in registers by one warp, element i = lane * PER + j in v[j]
// (PER a power of two): exchanges at distance >= PER go through shuffles, the shorter ones stay in the lane.
template <typename T>
__device__ __forceinline__ T warp_shfl_xor_key(T x, int m) {
    if constexpr (sizeof(T) == 8) {
        const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)x, m);
        const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(x >> 32), m);
        return ((T)hi << 32) | (T)lo;
    } else {
        return __shfl_xor_sync(0xffffffffu, x, m);
    }
}
template <int PER, typename T>
__device__ __forceinline__ void warp_sort_regs_desc(T (&v)[PER]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32 * PER; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= PER) {
                const int lx = stride / PER;
                const bool lower = (lane & lx) == 0;
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    const T o = warp_shfl_xor_key(v[j], lx);
                    const bool desc = ((lane * PER + j) & size) == 0;
                    // the lower index of a pair keeps the larger key in a descending block, the smaller otherwise
                    v[j] = (lower == desc) ? (v[j] > o ? v[j] : o) : (v[j] < o ? v[j] : o);
                }
            } else {
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    if (j & stride) continue;
                    const int j2 = j | stride;
                    const bool desc = ((lane * PER + j) & size) == 0;
                    const T a = v[j], b = v[j2];
                    if (desc ? (a < b) : (a > b)) {
                        v[j] = b;
                        v[j2] = a;
                    }
                }
            }
        }
    }
}

// Descending bitonic sort of kp keys (kp a power of two, kp <= blockDim.x) held one per thread, thread t holding
// position t (threads t >= kp hold 0 and keep 0); exchanges at distances below 32 go through warp shuffles, longer ones
// through `buf` (kp words of shared memory) with a barrier on each side.  Every thread of the block calls it.
__device__ __forceinline__ unsigned long long block_bitonic_desc_u64(unsigned long long v, int kp,
                                                                     unsigned long long* buf) {
    const int tid = threadIdx.x;
    for (int size = 2; size <= kp; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            unsigned long long o;
            if (stride >= 32) {
                if (tid < kp) buf[tid] = v;
                __syncthreads();
                o = tid < kp ? buf[tid ^ stride] : 0ull;
                __syncthreads();
            } else {
                const uint32_t lo = __shfl_xor_sync(0xffffffffu, (uint32_t)v, stride);
                const uint32_t hi = __shfl_xor_sync(0xffffffffu, (uint32_t)(v >> 32), stride);
                o = ((unsigned long long)hi << 32) | lo;
            }
            const bool desc = (tid & size) == 0, lower = (tid & stride) == 0;
            v = (lower == desc) ? (v > o ? v : o) : (v < o ? v : o);
        }
    }
    return tid < kp ? v : 0ull;
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block-wide sum of an int (all threads call; every thread gets the total).
__device__ __forceinline__ int block_sum_int(int v, int* red /* >= 32 ints of shared memory */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    int t = 0;
    for (int w = 0; w < nw; w++) t += red[w];
    __syncthreads();
    return t;
}

// In-place descending bitonic sort of n (a power of two) 64-bit keys in shared memory.
__device__ __forceinline__ void block_bitonic_desc(unsigned long long* a, int n) {
    const int tid = threadIdx.x, nt = blockDim.x;
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < n; i += nt) {
                int ixj = i ^ j;
                if (ixj > i) {
                    unsigned long long x = a[i], y = a[ixj];
                    bool desc = (i & k) == 0;
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace fvs
