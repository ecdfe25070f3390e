// Ex-code refinement, vanguard threshold and final top-k kernels.
//
//  refine_kernel     ex = f_add_ex + g + f_rescale_ex * (<q', 128 b + u> + kb)
//                    (reference: src/search/cpu_refinement.cpp:183-191 with the 7-bit code
//                     layout of third_party/rabitq/.../quantization/pack_excode.hpp:216-264,
//                     decoded as utils/space.hpp:677-762 does)
//  threshold_kernel  T1 = min(T0, k-th smallest seed distance)  (reference: vanguard seeds
//                    set thresholds, src/search/filter_kernels.cuh:308-468)
//  merge_kernel      best k by (ex, id) among ex < T0, padded with (FLT_MAX, 0)
//                    (reference: src/search/cpu_refinement.cpp:197-230,269-283)
#pragma once
#include <cfloat>

#include "common.cuh"
#include "kernels_scan.cuh"

namespace cora {

constexpr int kRefineThreads = 256;

struct ProbeInfo {  // per (query, probe rank), staged in shared memory by refine_kernel
    uint32_t start, size;
    float g;
};

// Inner product of the full 8-bit code of one vector with the rotated query x (in shared
// memory): lane l accumulates dims 64b+l and 64b+32+l of every 64-dim block b in fp64
// (exact products); this returns the lane's partial sum, and an xor butterfly over the
// warp (lane_sum) combines the lanes so that every lane holds the total.
__device__ __forceinline__ double code_ip_partial(const float *__restrict__ x,
                                                  const uint4 *code_base, uint32_t n,
                                                  const uint8_t *ex, int nblocks, int lane) {
    double acc = 0.0;
    for (int b = 0; b < nblocks; ++b) {
        const uint4 cw = __ldg(code_base + (size_t)(b >> 1) * n);
        const uint32_t w0 = (b & 1) ? cw.z : cw.x;
        const uint32_t w1 = (b & 1) ? cw.w : cw.y;
        const uint8_t *p = ex + 56 * b;
        const unsigned long long top = __ldg(reinterpret_cast<const unsigned long long *>(p + 48));
        uint32_t u0 = __ldg(p + lane) & 63u;
        uint32_t u1;
        if (lane < 16) {
            u1 = __ldg(p + 32 + lane) & 63u;
        } else {
            const int k = lane - 16;
            u1 = (static_cast<uint32_t>(__ldg(p + k)) >> 6) |
                 ((static_cast<uint32_t>(__ldg(p + 16 + k)) >> 6) << 2) |
                 ((static_cast<uint32_t>(__ldg(p + 32 + k)) >> 6) << 4);
        }
        u0 |= static_cast<uint32_t>((top >> (8 * (lane & 7) + (lane >> 3))) & 1ull) << 6;
        u1 |= static_cast<uint32_t>((top >> (8 * (lane & 7) + 4 + (lane >> 3))) & 1ull) << 6;
        const uint32_t b0 = (w0 >> (31 - lane)) & 1u, b1 = (w1 >> (31 - lane)) & 1u;
        acc = __fma_rn((double)x[64 * b + lane], (double)(128u * b0 + u0), acc);
        acc = __fma_rn((double)x[64 * b + 32 + lane], (double)(128u * b1 + u1), acc);
    }
    return acc;
}

__device__ __forceinline__ double lane_sum(double acc) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
        acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    return acc;
}

constexpr int kRefineInFlight = 4;  // candidates per warp whose loads overlap

// One CTA per query; warp per candidate, kRefineInFlight candidates in flight per warp.
// mode 0 refines the vanguard seeds [0, cnt) and records the seed count; mode 1 refines the
// main candidates [seed_cnt, cnt). Dynamic shared memory: D floats + nprobe ProbeInfo.
__global__ void __launch_bounds__(kRefineThreads) refine_kernel(IndexView ix, SearchView sv,
                                                                int mode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *x = reinterpret_cast<float *>(smem_raw);
    ProbeInfo *pinfo = reinterpret_cast<ProbeInfo *>(x + ix.D);
    const int q = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int kWarps = kRefineThreads / 32;
    const uint32_t cnt = sv.cand_cnt[q];
    const uint32_t cap = static_cast<uint32_t>(sv.cap);
    uint32_t from, to;
    if (mode == 0) {
        from = 0;
        to = min(cnt, cap);
        if (threadIdx.x == 0) sv.seed_cnt[q] = to;
    } else {
        from = sv.seed_cnt[q];
        to = min(cnt, cap);
    }
    if (from >= to) return;  // uniform across the block
    for (int j = threadIdx.x; j < ix.D; j += blockDim.x) x[j] = sv.qr[(size_t)q * ix.D + j];
    const int np = mode == 0 ? sv.veff : sv.nprobe;
    for (int r = threadIdx.x; r < np; r += blockDim.x) {
        const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
        pinfo[r] = ProbeInfo{ix.cl_start[c], ix.cl_size[c], sv.probe_g[(size_t)q * sv.nprobe + r]};
    }
    __syncthreads();
    const float kb = sv.scal[q].kb;
    const int nblocks = ix.D / 64;
    const size_t planes_per = static_cast<size_t>(ix.G16 + 1);
    for (uint32_t i0 = from + warp; i0 < to; i0 += kRefineInFlight * kWarps) {
        uint32_t idx[kRefineInFlight], gid[kRefineInFlight];
        ProbeInfo pi[kRefineInFlight];
        double part[kRefineInFlight];
#pragma unroll
        for (int t = 0; t < kRefineInFlight; ++t) {
            idx[t] = min(i0 + t * kWarps, to - 1);  // duplicates of the last one are not stored
            const uint64_t rec = sv.cand_rec[(size_t)q * sv.cap + idx[t]];
            gid[t] = static_cast<uint32_t>(rec & 0xFFFFFFFFu);
            pi[t] = pinfo[rec >> 32];
        }
#pragma unroll
        for (int t = 0; t < kRefineInFlight; ++t)
            part[t] = code_ip_partial(x, ix.scan4 + planes_per * pi[t].start + (gid[t] - pi[t].start),
                                      pi[t].size, ix.long_codes + (size_t)gid[t] * ix.LC, nblocks,
                                      lane);
#pragma unroll
        for (int t = 0; t < kRefineInFlight; ++t) {
            const double ip = lane_sum(part[t]);
            if (lane == 0 && i0 + t * kWarps < to) {
                const float2 f = ix.ex_factors[gid[t]];
                const float ex_d = __fadd_rn(__fadd_rn(f.x, pi[t].g),
                                             __fmul_rn(f.y, __fadd_rn(__double2float_rn(ip), kb)));
                sv.cand_key[(size_t)q * sv.cap + idx[t]] = make_key(ex_d, ix.ids[gid[t]]);
            }
        }
    }
}

// One CTA per query: T1 = min(T0, k-th smallest seed distance below T0) when at least k
// seeds are below T0, else T0. Dynamic shared memory: next_pow2(k) keys.
__global__ void __launch_bounds__(256) threshold_kernel(SearchView sv) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    const int q = blockIdx.x;
    const float T0 = sv.T0[q];
    const uint32_t n = sv.seed_cnt[q];
    const uint64_t *keys = sv.cand_key + (size_t)q * sv.cap;
    auto key_at = [&](uint32_t i) -> uint64_t {
        const uint64_t key = keys[i];
        return unord_f32(static_cast<uint32_t>(key >> 32)) < T0 ? key : kKeyMax;
    };
    block_select_smallest(key_at, n, sv.k, s_keys, scratch);
    if (threadIdx.x == 0) {
        const uint64_t kth = s_keys[sv.k - 1];
        sv.T1[q] = kth == kKeyMax ? T0 : fminf(T0, unord_f32(static_cast<uint32_t>(kth >> 32)));
    }
}

// One CTA per query: final top-k by (ex, id) among all refined candidates with ex < T0.
// Writes distances / ids (padded with FLT_MAX / 0), records the query's threshold after the
// search (its k-th distance when k results exist, else T0; what capture_thresholds()
// reports) and adds the candidate count to stats[0]. Dynamic shared memory: next_pow2(k).
__global__ void __launch_bounds__(256) merge_kernel(SearchView sv, float *__restrict__ out_d,
                                                    uint32_t *__restrict__ out_i,
                                                    unsigned long long *__restrict__ stats) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    const int q = blockIdx.x;
    const float T0 = sv.T0[q];
    const uint32_t cnt = sv.cand_cnt[q];
    const uint32_t n = min(cnt, static_cast<uint32_t>(sv.cap));
    const uint64_t *keys = sv.cand_key + (size_t)q * sv.cap;
    auto key_at = [&](uint32_t i) -> uint64_t {
        const uint64_t key = keys[i];
        return unord_f32(static_cast<uint32_t>(key >> 32)) < T0 ? key : kKeyMax;
    };
    block_select_smallest(key_at, n, sv.k, s_keys, scratch);
    for (int j = threadIdx.x; j < sv.k; j += blockDim.x) {
        const uint64_t key = s_keys[j];
        const bool ok = key != kKeyMax;
        out_d[(size_t)q * sv.k + j] = ok ? unord_f32(static_cast<uint32_t>(key >> 32)) : FLT_MAX;
        out_i[(size_t)q * sv.k + j] = ok ? static_cast<uint32_t>(key & 0xFFFFFFFFu) : 0u;
    }
    if (threadIdx.x == 0) {
        const uint64_t kth = s_keys[sv.k - 1];
        sv.Tcap[q] = kth != kKeyMax ? unord_f32(static_cast<uint32_t>(kth >> 32)) : T0;
        atomicAdd(stats, static_cast<unsigned long long>(cnt));
    }
}

}  // namespace cora
