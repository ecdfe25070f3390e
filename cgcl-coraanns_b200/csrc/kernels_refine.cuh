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

constexpr int kRefineThreads = 128;

struct ProbeInfo {  // per (query, probe rank), staged in shared memory by refine_kernel
    uint32_t start, size;
    float g;
};

// One 64-dim block of the full 8-bit code inner product, continuing the fp64 chain `acc`
// in ascending dimension order (every product is exact in fp64). `e` holds the block's 56
// ex-code bytes (pack_excode.hpp:216-264 layout: bytes 0..47 carry the low 6 bits of dims
// 0..47 and 2-bit slices of dims 48..63, bytes 48..55 the top bits), w0 / w1 the 1-bit
// code words of dims 0..31 / 32..63, x the block's 64 rotated query values.
__device__ __forceinline__ double block_code_ip(const float *__restrict__ x, const uint64_t (&e)[7],
                                                uint32_t w0, uint32_t w1, double acc) {
#pragma unroll
    for (int d = 0; d < 64; ++d) {
        uint32_t u;
        if (d < 48) {
            u = static_cast<uint32_t>(e[d >> 3] >> (8 * (d & 7))) & 63u;
        } else {
            const int k = d - 48;
            const uint32_t b0 = static_cast<uint32_t>(e[k >> 3] >> (8 * (k & 7))) & 0xFFu;
            const uint32_t b1 = static_cast<uint32_t>(e[(16 + k) >> 3] >> (8 * ((16 + k) & 7))) & 0xFFu;
            const uint32_t b2 = static_cast<uint32_t>(e[(32 + k) >> 3] >> (8 * ((32 + k) & 7))) & 0xFFu;
            u = (b0 >> 6) | ((b1 >> 6) << 2) | ((b2 >> 6) << 4);
        }
        u |= static_cast<uint32_t>((e[6] >> (8 * (d & 7) + (d >> 3))) & 1ull) << 6;
        const uint32_t w = d < 32 ? w0 : w1;
        const uint32_t bit = (w >> (31 - (d & 31))) & 1u;
        acc = __fma_rn((double)x[d], (double)(128u * bit + u), acc);
    }
    return acc;
}

// One CTA per query, one thread per candidate: every load of a candidate (1-bit code words,
// ex code, factors, id) is issued before its fp64 chain, so a candidate costs one memory
// round trip. mode 0 refines the vanguard seeds [0, cnt) and records the seed count; mode 1
// refines the main candidates [seed_cnt, cnt). Dynamic shared memory: D floats + nprobe
// ProbeInfo.
__global__ void __launch_bounds__(kRefineThreads) refine_kernel(IndexView ix, SearchView sv,
                                                                int mode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float *x = reinterpret_cast<float *>(smem_raw);
    ProbeInfo *pinfo = reinterpret_cast<ProbeInfo *>(x + ix.D);
    const int q = blockIdx.x;
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
    for (uint32_t i = from + threadIdx.x; i < to; i += blockDim.x) {
        const uint64_t rec = sv.cand_rec[(size_t)q * sv.cap + i];
        const uint32_t gid = static_cast<uint32_t>(rec & 0xFFFFFFFFu);
        const ProbeInfo p = pinfo[rec >> 32];
        const uint4 *cb = ix.scan4 + planes_per * p.start + (gid - p.start);
        const uint64_t *eb = reinterpret_cast<const uint64_t *>(ix.long_codes + (size_t)gid * ix.LC);
        const float2 f = __ldg(ix.ex_factors + gid);
        const uint32_t id = __ldg(ix.ids + gid);
        double acc = 0.0;
        for (int g = 0; 2 * g < nblocks; ++g) {
            const uint4 cw = __ldg(cb + (size_t)g * p.size);
            uint64_t e[7];
#pragma unroll
            for (int t = 0; t < 7; ++t) e[t] = __ldg(eb + 14 * g + t);
            acc = block_code_ip(x + 128 * g, e, cw.x, cw.y, acc);
            if (2 * g + 1 < nblocks) {
#pragma unroll
                for (int t = 0; t < 7; ++t) e[t] = __ldg(eb + 14 * g + 7 + t);
                acc = block_code_ip(x + 128 * g + 64, e, cw.z, cw.w, acc);
            }
        }
        const float ex_d = __fadd_rn(__fadd_rn(f.x, p.g),
                                     __fmul_rn(f.y, __fadd_rn(__double2float_rn(acc), kb)));
        sv.cand_key[(size_t)q * sv.cap + i] = make_key(ex_d, id);
    }
}

__device__ __forceinline__ float threshold_from_kth(uint64_t kth, float T0) {
    return kth == kKeyMax ? T0 : fminf(T0, unord_f32(static_cast<uint32_t>(kth >> 32)));
}

// Writes a query's k selected keys as its final result: distances / ids padded with
// (FLT_MAX, 0), and the threshold after the search (k-th distance when k results exist,
// else T0; what capture_thresholds() reports).
__device__ __forceinline__ void write_topk(const uint64_t *s_keys, int q, int k, float T0,
                                           float *out_d, uint32_t *out_i, float *Tcap) {
    for (int j = threadIdx.x; j < k; j += blockDim.x) {
        const uint64_t key = s_keys[j];
        const bool ok = key != kKeyMax;
        out_d[(size_t)q * k + j] = ok ? unord_f32(static_cast<uint32_t>(key >> 32)) : FLT_MAX;
        out_i[(size_t)q * k + j] = ok ? static_cast<uint32_t>(key & 0xFFFFFFFFu) : 0u;
    }
    if (threadIdx.x == 0) {
        const uint64_t kth = s_keys[k - 1];
        Tcap[q] = kth != kKeyMax ? unord_f32(static_cast<uint32_t>(kth >> 32)) : T0;
    }
}

// One CTA per query: T1 = min(T0, k-th smallest seed distance below T0) when at least k
// seeds are below T0, else T0. Sharded search (keys_out != nullptr): writes this shard's k
// smallest seed keys (padded with kKeyMax) to keys_out[q * k ..] instead, for the exchange;
// gather_threshold_kernel then derives T1 from every shard's keys. Dynamic shared memory:
// next_pow2(k) keys.
__global__ void __launch_bounds__(256) threshold_kernel(SearchView sv,
                                                        uint64_t *__restrict__ keys_out) {
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
    if (keys_out) {
        for (int j = threadIdx.x; j < sv.k; j += blockDim.x)
            keys_out[(size_t)q * sv.k + j] = s_keys[j];
    } else if (threadIdx.x == 0) {
        sv.T1[q] = threshold_from_kth(s_keys[sv.k - 1], T0);
    }
}

// One CTA per query: final top-k by (ex, id) among all refined candidates with ex < T0, and
// the candidate count added to stats[0]. keys_out == nullptr: writes the result
// (write_topk). Sharded search: writes this shard's k best keys to keys_out[q * k ..] and,
// from block 0, the shard's device error word to keys_out[nq * k], for the exchange that
// gather_merge_kernel completes. Dynamic shared memory: next_pow2(k).
__global__ void __launch_bounds__(256) merge_kernel(SearchView sv, float *__restrict__ out_d,
                                                    uint32_t *__restrict__ out_i,
                                                    unsigned long long *__restrict__ stats,
                                                    uint64_t *__restrict__ keys_out) {
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
    if (keys_out) {
        for (int j = threadIdx.x; j < sv.k; j += blockDim.x)
            keys_out[(size_t)q * sv.k + j] = s_keys[j];
        if (q == 0 && threadIdx.x == 0)
            keys_out[(size_t)sv.nq * sv.k] = static_cast<uint32_t>(*sv.err);
    } else {
        write_topk(s_keys, q, sv.k, T0, out_d, out_i, sv.Tcap);
    }
    if (threadIdx.x == 0) atomicAdd(stats, static_cast<unsigned long long>(cnt));
}

// ---- shard exchange (cluster-sharded search) -----------------------------------------
// `recv` holds `world` blocks of `stride` u64 (stride = nq * k + 1), block r = shard r's
// exchange buffer: k keys per query, then one word (a device error word in the final
// exchange). One CTA per query; dynamic shared memory: next_pow2(k) keys.

// T1 = min(T0, k-th smallest seed key over every shard) (the single-GPU threshold_kernel
// over the union of the shards' seeds, which contains the k smallest).
__global__ void __launch_bounds__(256) gather_threshold_kernel(const uint64_t *__restrict__ recv,
                                                               int world, size_t stride,
                                                               SearchView sv) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    const int q = blockIdx.x;
    const int k = sv.k;
    auto key_at = [&](uint32_t i) -> uint64_t {
        const uint32_t r = i / static_cast<uint32_t>(k), j = i - r * static_cast<uint32_t>(k);
        return recv[r * stride + (size_t)q * k + j];
    };
    block_select_smallest(key_at, static_cast<uint32_t>(world * k), k, s_keys, scratch);
    if (threadIdx.x == 0) sv.T1[q] = threshold_from_kth(s_keys[k - 1], sv.T0[q]);
}

// Final top-k over every shard's k best keys; ORs every shard's error word into sv.err so
// that each rank reports a failure on any shard.
__global__ void __launch_bounds__(256) gather_merge_kernel(const uint64_t *__restrict__ recv,
                                                           int world, size_t stride,
                                                           SearchView sv, float *__restrict__ out_d,
                                                           uint32_t *__restrict__ out_i) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    const int q = blockIdx.x;
    const int k = sv.k;
    auto key_at = [&](uint32_t i) -> uint64_t {
        const uint32_t r = i / static_cast<uint32_t>(k), j = i - r * static_cast<uint32_t>(k);
        return recv[r * stride + (size_t)q * k + j];
    };
    block_select_smallest(key_at, static_cast<uint32_t>(world * k), k, s_keys, scratch);
    write_topk(s_keys, q, k, sv.T0[q], out_d, out_i, sv.Tcap);
    if (q == 0 && threadIdx.x == 0) {
        uint32_t e = 0;
        for (int r = 0; r < world; ++r) e |= static_cast<uint32_t>(recv[r * stride + stride - 1]);
        if (e) atomicOr(sv.err, static_cast<int>(e));
    }
}

}  // namespace cora
