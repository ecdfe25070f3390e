// Shared device utilities for the IVF-RaBitQ search kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace cora {

// ---- ordering ------------------------------------------------------------------------
// Monotone float -> uint32 map; every (value, id) order in the search contract is the
// lexicographic order of (ord_f32(value), id) packed as a uint64 key.
__host__ __device__ __forceinline__ uint32_t ord_f32(float f) {
#ifdef __CUDA_ARCH__
    const uint32_t u = __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, 4);
#endif
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ __forceinline__ float unord_f32(uint32_t o) {
    const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    __builtin_memcpy(&f, &u, 4);
    return f;
#endif
}
__host__ __device__ __forceinline__ uint64_t make_key(float v, uint32_t id) {
    return (static_cast<uint64_t>(ord_f32(v)) << 32) | id;
}
constexpr uint64_t kKeyMax = ~0ull;

// ---- device error word ---------------------------------------------------------------
// Kernels never trap; a bounded wait that gives up, or a capacity overflow, sets a bit
// here and the host turns it into an error after the stream synchronises.
enum DeviceError : int {
    kDevOk = 0,
    kDevCandidateOverflow = 1,
    kDevWaitTimeout = 2,
    kDevBadInput = 4,
};

// ---- TMA bulk copies (cp.async.bulk into this CTA's shared memory only) with bounded
// mbarrier waits ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Waits for the mbarrier phase with a wall-clock limit (default 2 s). On timeout it
// records kDevWaitTimeout and returns false; the caller stops issuing work and exits.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err,
                                                  uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit_ns) {
            atomicOr(err, kDevWaitTimeout);
            return false;
        }
        __nanosleep(64);
    }
}
// 1-D bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes,
                                         uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---- block-wide bitonic sort of a power-of-two uint64 array in shared memory ---------
// Callers synchronise before the call; the function ends with a barrier.
__device__ __forceinline__ void block_bitonic_sort(uint64_t *a, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t x = a[i], y = a[ixj];
                    const bool up = (i & k) == 0;
                    if ((x > y) == up) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Row stride (floats) of the probe GEMM's per-chunk row minima: ceil(nlist / 32) rounded up
// to a multiple of 8 (8 chunks of 32 columns per 256-column tile).
__host__ __device__ __forceinline__ int chunk_stride(int nlist) { return (nlist + 255) / 256 * 8; }

// Inclusive prefix sum over the lanes of a full warp.
__device__ __forceinline__ uint32_t warp_inclusive_sum(uint32_t v, int lane) {
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += o;
    }
    return v;
}

// ---- warp-wide bitonic sorts of uint64 keys -----------------------------------------------
// One key per lane, returned ascending by lane index.
__device__ __forceinline__ uint64_t warp_sort_lane_keys(uint64_t v, int lane) {
    for (int k = 2; k <= 32; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            const uint64_t o = __shfl_xor_sync(0xffffffffu, v, j);
            const bool up = (lane & k) == 0, lower = (lane & j) == 0;
            v = (lower == up) ? (v < o ? v : o) : (v < o ? o : v);
        }
    }
    return v;
}

// n (a power of two) keys in shared memory, sorted ascending by the calling warp.
__device__ __forceinline__ void warp_sort_smem(uint64_t *a, int n, int lane) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const uint64_t x = a[i], y = a[ixj];
                    if ((x > y) == ((i & k) == 0)) {
                        a[i] = y;
                        a[ixj] = x;
                    }
                }
            }
            __syncwarp();
        }
    }
}

__host__ __device__ __forceinline__ int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

// ---- block-wide radix selection of the S smallest uint64 keys ------------------------
// Keys are unique (an id sits in the low 32 bits); kKeyMax marks an item filtered out.
// MSB-first passes over 8-bit digits narrow the prefix of the S-th smallest key, stopping
// as soon as the digit bucket holding it is taken whole. The selected keys are written to
// out[0, S) in ascending order (kKeyMax where fewer than S exist). `key_at(i)` yields key i
// of n; `scratch` is 256 + 3 ints of shared memory; out holds next_pow2(S) keys.
// All threads of the block must call this function.
template <typename KeyAt>
__device__ void block_select_smallest(KeyAt key_at, uint32_t n, int S, uint64_t *out,
                                      int *scratch) {
    int *hist = scratch;            // 256 bins
    int *s_sel = scratch + 256;     // [0] chosen digit, [1] rank in bin / cursor, [2] bin size
    const int tid = threadIdx.x;
    const int S2 = next_pow2(S);
    for (int i = tid; i < S2; i += blockDim.x) out[i] = kKeyMax;
    uint64_t prefix = 0;            // digits fixed so far
    int shift = 64;                 // keys match prefix on bits >= shift
    uint32_t rank = static_cast<uint32_t>(S);  // 1-based rank still to locate
    bool take_all = n <= static_cast<uint32_t>(S);
    while (!take_all && shift > 0) {
        shift -= 8;
        for (int b = tid; b < 256; b += blockDim.x) hist[b] = 0;
        __syncthreads();
        for (uint32_t i = tid; i < n; i += blockDim.x) {
            const uint64_t k = key_at(i);
            if (shift + 8 >= 64 || (k >> (shift + 8)) == (prefix >> (shift + 8)))
                atomicAdd(&hist[(k >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid < 32) {  // warp 0 scans the 256 bins (8 per lane) and picks the digit
            int local[8], sum = 0;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                local[t] = hist[tid * 8 + t];
                sum += local[t];
            }
            int incl = sum;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, off);
                if (tid >= off) incl += v;
            }
            int before = incl - sum;
            const bool mine = before < static_cast<int>(rank) && static_cast<int>(rank) <= incl;
            if (mine) {
                for (int t = 0; t < 8; ++t) {
                    if (before + local[t] >= static_cast<int>(rank)) {
                        s_sel[0] = tid * 8 + t;
                        s_sel[1] = static_cast<int>(rank) - before;  // rank inside the bin
                        s_sel[2] = local[t];
                        break;
                    }
                    before += local[t];
                }
            }
        }
        __syncthreads();
        const int digit = s_sel[0];
        const int in_bin = s_sel[1];
        const int bin_size = s_sel[2];
        __syncthreads();
        prefix |= static_cast<uint64_t>(digit) << shift;
        rank = static_cast<uint32_t>(in_bin);
        if (in_bin == bin_size) take_all = true;  // the whole bucket is selected
    }
    // Select every key whose bits >= shift are <= prefix's (all keys when take_all && n<=S).
    if (tid == 0) s_sel[1] = 0;
    __syncthreads();
    const bool everything = n <= static_cast<uint32_t>(S);
    for (uint32_t i = tid; i < n; i += blockDim.x) {
        const uint64_t k = key_at(i);
        const bool sel = everything || (shift >= 64 ? true : (k >> shift) <= (prefix >> shift));
        if (sel) {
            const int pos = atomicAdd(&s_sel[1], 1);
            if (pos < S) out[pos] = k;
        }
    }
    __syncthreads();
    block_bitonic_sort(out, S2);
}


// Streaming block top-S of uint64 keys (ascending). Shared layout: buf[0, S) holds the
// current best (sorted; unused slots kKeyMax), buf[S, S + stage_cap) stages new keys,
// buf is sized `sort_n` = next_pow2(S + stage_cap). Keys must be < threshold() to be
// staged; at most stage_cap keys may be staged between two flush() calls.
struct BlockTopK {
    uint64_t *buf;
    int S, stage_cap, sort_n;
    int *n_staged;      // shared counter
    uint64_t *thresh;   // shared: current S-th best key (kKeyMax while fewer than S)

    __device__ void init(uint64_t limit_key) {
        for (int i = threadIdx.x; i < sort_n; i += blockDim.x) buf[i] = kKeyMax;
        if (threadIdx.x == 0) {
            *n_staged = 0;
            *thresh = limit_key;
        }
        __syncthreads();
    }
    __device__ __forceinline__ void offer(uint64_t key) {
        if (key < *thresh) {
            const int pos = atomicAdd(n_staged, 1);
            buf[S + pos] = key;
        }
    }
    // All threads call after their offers. `limit_key` caps the threshold (strict bound).
    __device__ void flush(uint64_t limit_key) {
        __syncthreads();
        const int n = *n_staged;
        if (n == 0) return;
        // Only the occupied prefix is sorted: [S + n, m) is padded with kKeyMax and every
        // slot at or beyond m already holds kKeyMax.
        const int m = next_pow2(S + n);
        for (int i = S + n + threadIdx.x; i < m; i += blockDim.x) buf[i] = kKeyMax;
        __syncthreads();
        block_bitonic_sort(buf, m);
        if (threadIdx.x == 0) {
            *n_staged = 0;
            const uint64_t t = buf[S - 1];
            *thresh = t < limit_key ? t : limit_key;
        }
        __syncthreads();
    }
};

}  // namespace cora
