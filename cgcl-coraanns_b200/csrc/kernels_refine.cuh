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

// One CTA per query; warp per candidate. mode 0 refines the vanguard seeds [0, cnt) and
// records the seed count; mode 1 refines the main candidates [seed_cnt, cnt).
// The 8-bit-code inner product accumulates in fp64: lane l owns dims 64b+l and 64b+32+l
// of every 64-dim block b (ascending), then an xor butterfly combines the lanes.
__global__ void __launch_bounds__(kRefineThreads) refine_kernel(IndexView ix, SearchView sv,
                                                                int mode) {
    const int q = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
    const float kb = sv.scal[q].kb;
    const float *x = sv.qr + (size_t)q * ix.D;
    const int nblocks = ix.D / 64;
    const int G16 = ix.G16;
    for (uint32_t i = from + warp; i < to; i += kRefineThreads / 32) {
        const uint64_t rec = sv.cand_rec[(size_t)q * sv.cap + i];
        const uint32_t gid = static_cast<uint32_t>(rec & 0xFFFFFFFFu);
        const int r = static_cast<int>(rec >> 32);
        const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
        const float g = sv.probe_g[(size_t)q * sv.nprobe + r];
        const uint32_t s = ix.cl_start[c];
        const uint32_t n = ix.cl_size[c];
        const uint32_t iv = gid - s;
        const uint4 *code_base = ix.scan4 + (size_t)(G16 + 1) * s + iv;
        const uint8_t *ex = ix.long_codes + (size_t)gid * ix.LC;
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
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
            acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
        if (lane == 0) {
            const float ipt = __double2float_rn(acc);
            const float2 f = ix.ex_factors[gid];
            const float ex_d = __fadd_rn(__fadd_rn(f.x, g), __fmul_rn(f.y, __fadd_rn(ipt, kb)));
            sv.cand_key[(size_t)q * sv.cap + i] = make_key(ex_d, ix.ids[gid]);
        }
    }
}

constexpr int kMergeTile = 1024;

// One CTA per query: T1 = min(T0, k-th smallest seed distance below T0) when at least k
// seeds are below T0, else T0. Dynamic shared memory: sort_n = next_pow2(k + 1024) keys.
__global__ void __launch_bounds__(256) threshold_kernel(SearchView sv, int sort_n) {
    extern __shared__ uint64_t smem_k[];
    __shared__ int n_staged;
    __shared__ uint64_t thresh;
    const int q = blockIdx.x;
    const float T0 = sv.T0[q];
    const uint32_t n = sv.seed_cnt[q];
    BlockTopK tk{smem_k, sv.k, kMergeTile, sort_n, &n_staged, &thresh};
    tk.init(kKeyMax);
    for (uint32_t base = 0; base < n; base += kMergeTile) {
        for (uint32_t i = base + threadIdx.x; i < min(n, base + kMergeTile); i += blockDim.x) {
            const uint64_t key = sv.cand_key[(size_t)q * sv.cap + i];
            if (unord_f32(static_cast<uint32_t>(key >> 32)) < T0) tk.offer(key);
        }
        tk.flush(kKeyMax);
    }
    if (threadIdx.x == 0) {
        const uint64_t kth = smem_k[sv.k - 1];
        sv.T1[q] = kth == kKeyMax ? T0 : fminf(T0, unord_f32(static_cast<uint32_t>(kth >> 32)));
    }
}

// One CTA per query: final top-k by (ex, id) among all refined candidates with ex < T0.
// Writes distances / ids (padded with FLT_MAX / 0), records the query's threshold after the
// search (its k-th distance when k results exist, else T0; what capture_thresholds()
// reports) and adds the candidate count to stats[0].
__global__ void __launch_bounds__(256) merge_kernel(SearchView sv, int sort_n,
                                                    float *__restrict__ out_d,
                                                    uint32_t *__restrict__ out_i,
                                                    unsigned long long *__restrict__ stats) {
    extern __shared__ uint64_t smem_k[];
    __shared__ int n_staged;
    __shared__ uint64_t thresh;
    const int q = blockIdx.x;
    const float T0 = sv.T0[q];
    const uint32_t cnt = sv.cand_cnt[q];
    const uint32_t n = min(cnt, static_cast<uint32_t>(sv.cap));
    BlockTopK tk{smem_k, sv.k, kMergeTile, sort_n, &n_staged, &thresh};
    tk.init(kKeyMax);
    for (uint32_t base = 0; base < n; base += kMergeTile) {
        for (uint32_t i = base + threadIdx.x; i < min(n, base + kMergeTile); i += blockDim.x) {
            const uint64_t key = sv.cand_key[(size_t)q * sv.cap + i];
            if (unord_f32(static_cast<uint32_t>(key >> 32)) < T0) tk.offer(key);
        }
        tk.flush(kKeyMax);
    }
    for (int j = threadIdx.x; j < sv.k; j += blockDim.x) {
        const uint64_t key = smem_k[j];
        const bool ok = key != kKeyMax;
        out_d[(size_t)q * sv.k + j] = ok ? unord_f32(static_cast<uint32_t>(key >> 32)) : FLT_MAX;
        out_i[(size_t)q * sv.k + j] = ok ? static_cast<uint32_t>(key & 0xFFFFFFFFu) : 0u;
    }
    if (threadIdx.x == 0) {
        const uint64_t kth = smem_k[sv.k - 1];
        sv.Tcap[q] = kth != kKeyMax ? unord_f32(static_cast<uint32_t>(kth >> 32)) : T0;
        atomicAdd(stats, static_cast<unsigned long long>(cnt));
    }
}

}  // namespace cora
