// Ex-code refinement, vanguard threshold and final top-k kernels.
//
//  refine_kernel     ex = (f_add_ex + g) + f_rescale_ex * ((128 ip1 + ip2) + kb), with
//                    ip1 = width * ip_int the scan's integer estimate of <q', b> and
//                    ip2 = <q', u> (reference: src/search/cpu_refinement.cpp:183-191 =
//                    split_distance_boosting, third_party/rabitq/.../index/estimator.hpp:
//                    86-103, with the 7-bit code layout of quantization/pack_excode.hpp:
//                    216-264, decoded as utils/space.hpp:677-762 does); opt-in full-code
//                    form: (f_add_ex + g) + f_rescale_ex * (<q', 128 b + u> + kb)
//  threshold_kernel  T1 = min(T0, k-th smallest seed distance)  (reference: vanguard seeds
//                    set thresholds, src/search/filter_kernels.cuh:308-468)
//  merge_kernel      best k by (ex, id) among ex < T0, padded with (FLT_MAX, 0)
//                    (reference: src/search/cpu_refinement.cpp:197-230,269-283)
#pragma once
#include <cfloat>

#include "common.cuh"
#include "kernels_scan.cuh"

namespace cora {

#ifndef CORA_REFINE_THREADS
#define CORA_REFINE_THREADS 128
#endif
// threads per query in refine_kernel; measured on config 2 (candidate refine): 64 -> 0.202
// ms, 128 -> 0.192, 256 -> 0.188 (seed refine 0.080 / 0.072 / 0.075)
constexpr int kRefineThreads = CORA_REFINE_THREADS;

struct ProbeInfo {  // per (query, probe rank), staged in shared memory by refine_kernel
    uint32_t start, size;
    float g;  // the additive query term g_add
};

// The 8-bit codes c = 128 b + u of dims d0 .. d0 + 3 of one 64-dim block, as the bytes of a
// word (SWAR). `ew` holds the block's 56 ex-code bytes (pack_excode.hpp:216-264 layout:
// bytes 0..47 carry the low 6 bits of dims 0..47 and 2-bit slices of dims 48..63, bytes
// 48..55 the top bits), rbits the bit-reversed 1-bit code word of the block's half that
// holds d0.
__device__ __forceinline__ uint32_t code4(const uint32_t (&ew)[14], uint32_t rbits, int d0) {
    uint32_t low;
    if (d0 < 48) {
        low = ew[d0 / 4] & 0x3F3F3F3Fu;  // low 6 bits of dims d0..d0+3 = bytes d0..d0+3
    } else {                             // dims 48 + k: top 2 bits of bytes k, 16 + k, 32 + k
        const int t = (d0 - 48) / 4;
        low = ((ew[t] >> 6) & 0x03030303u) | ((ew[4 + t] >> 4) & 0x0C0C0C0Cu) |
              ((ew[8 + t] >> 2) & 0x30303030u);
    }
    // bit 6: dim 8k + m sits at bit 8m + k of bytes 48..55 (word 12 for m < 4, else 13)
    const int k = d0 >> 3;
    const uint32_t top = ((ew[12 + ((d0 & 7) >> 2)] >> k) & 0x01010101u) << 6;
    // bit 7: the 1-bit code, dim d at bit (d & 31) of the bit-reversed word; spread the four
    // bits of dims d0..d0+3 to bit 7 of bytes 0..3 (the shifted copies do not overlap)
    const uint32_t nib = (rbits >> (d0 & 31)) & 0xFu;
    const uint32_t msb = (nib * 0x10204080u) & 0x80808080u;
    return low | top | msb;
}

// One CTA per cluster (clusters c0 + blockIdx.x), at load: the refine rows (the 8-bit codes
// c = 128 b + u of every dimension, decoded by code4 from the ex codes and the 1-bit code
// words in the scan planes) and the meta words {f_add_ex, f_rescale_ex, id, 0} of its
// vectors. long_codes / exf / ids hold a staged batch of whole clusters starting at vector v0.
__global__ void __launch_bounds__(256) build_refine_rows_kernel(
    const uint8_t *__restrict__ long_codes, const float2 *__restrict__ exf,
    const uint32_t *__restrict__ ids, const uint4 *__restrict__ scan4,
    const uint32_t *__restrict__ cl_start, const uint32_t *__restrict__ cl_size, int D, int G16,
    int LC, uint32_t c0, uint64_t v0, uint8_t *__restrict__ rows, uint4 *__restrict__ meta) {
    const uint32_t c = c0 + blockIdx.x;
    const uint32_t s = cl_start[c], n = cl_size[c];
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const size_t gid = (size_t)s + i, lid = gid - v0;
        uint32_t *row = reinterpret_cast<uint32_t *>(rows + gid * D);
        for (int blk = 0; blk < D / 64; ++blk) {
            // 56 ex-code bytes of the block (rows of LC = 7 D / 8 bytes: 8-byte aligned)
            const uint32_t *eb =
                reinterpret_cast<const uint32_t *>(long_codes + lid * LC + 56 * blk);
            uint32_t ew[14];
            for (int t = 0; t < 14; ++t) ew[t] = eb[t];
            const uint4 cw = scan4[(size_t)(G16 + 1) * s + (size_t)(blk / 2) * n + i];
            const uint32_t w0 = (blk & 1) ? cw.z : cw.x, w1 = (blk & 1) ? cw.w : cw.y;
            const uint32_t r0 = __brev(w0), r1 = __brev(w1);
            for (int d0 = 0; d0 < 64; d0 += 4)
                row[(64 * blk + d0) / 4] = code4(ew, d0 < 32 ? r0 : r1, d0);
        }
        const float2 f = exf[lid];
        meta[gid] = make_uint4(__float_as_uint(f.x), __float_as_uint(f.y), ids[lid], 0u);
    }
}

// Refinement forms: the reference's expression with ip1 from the integer estimator (the
// default) or from the LUT estimator (with the scan's estimator), or the full-code inner
// product (opt-in).
enum RefineForm : int { kRefineSplitInt = 0, kRefineSplitLut = 1, kRefineFullCode = 2 };

// One 64-dim block (index blk) of a refine row (v: its 64 codes c = 128 b + u, 4 per word,
// dimension order) against the rotated query x (fp64, shared memory), continuing the fp64
// chain `acc` in ascending dimension order (every product is exact in fp64). Each byte
// becomes the double c (or u = c & 127) exactly as (2^52 + c) - 2^52 from its bit pattern,
// so the loop runs no conversion instructions.
//   kRefineSplitInt: acc accumulates <x, u>, and ip accumulates sum_i b_i qint_i with dp4a
//     over the code words' top bits and the query's qint bytes (qw: qint of dims 4t .. 4t + 3
//     as the signed bytes of word t), exact in int32;
//   kRefineSplitLut: acc accumulates <x, u>, and la0 / la1 the LUT estimator's sums: row
//     word t (dims 4t .. 4t + 3) is nibble group t, whose pattern is the four code bits (dim
//     4t at bit 3); even groups go to la0, odd ones to la1, in ascending order (the scan's
//     order, ip_from_lut), from the fp32 tables T (16 per group);
//   kRefineFullCode: acc accumulates <x, 128 b + u>.
template <int kForm>
__device__ __forceinline__ void block_code8_ip(const double *__restrict__ x,
                                               const uint32_t *__restrict__ qw,
                                               const float *__restrict__ T, int blk,
                                               const uint4 (&v)[4], double &acc, int &ip,
                                               float &la0, float &la1) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t w4[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const uint32_t w = kForm == kRefineFullCode ? w4[h] : (w4[h] & 0x7F7F7F7Fu);
            if (kForm == kRefineSplitInt)
                ip = __dp4a(static_cast<int>((w4[h] >> 7) & 0x01010101u),
                            static_cast<int>(qw[16 * blk + 4 * t + h]), ip);
            if (kForm == kRefineSplitLut) {
                const uint32_t pat = ((w4[h] >> 4) & 8u) | ((w4[h] >> 13) & 4u) |
                                     ((w4[h] >> 22) & 2u) | (w4[h] >> 31);
                const float e = T[(16 * blk + 4 * t + h) * 16 + pat];
                if (h & 1)
                    la1 = __fadd_rn(la1, e);
                else
                    la0 = __fadd_rn(la0, e);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t c = __byte_perm(w, 0u, 0x4440u | i);
                const double cd = __dsub_rn(__hiloint2double(0x43300000, static_cast<int>(c)),
                                            4503599627370496.0);
                acc = __fma_rn(x[16 * t + 4 * h + i], cd, acc);
            }
        }
    }
}

__device__ __forceinline__ void load_block(uint4 (&v)[4], const uint4 *__restrict__ row, int blk) {
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] = __ldg(row + 4 * blk + u);
}

// The refinement of one candidate row: the factor t of f_rescale_ex. kPipelined (long rows,
// D > 128): the row's 64-byte blocks are loaded two ahead of the one being accumulated
// (three register buffers in rotation), so a thread keeps 128 bytes of its row in flight
// during the fp64 chain (measured at D = 768: 0.90 instead of 1.62 ms for 2000 queries x
// ~1500 candidates); at D <= 128 (two blocks per row) it gains nothing and its registers
// (168 instead of 40) cost occupancy, so those rows are loaded block by block.
template <int kForm, bool kPipelined>
__device__ __forceinline__ float refine_row_term(const uint4 *__restrict__ row, int nblocks,
                                                 const double *__restrict__ x,
                                                 const uint32_t *__restrict__ qw,
                                                 const float *__restrict__ T, float width,
                                                 float kb) {
    double acc = 0.0;
    int ip = 0;
    float la0 = 0.0f, la1 = 0.0f;
    if (kPipelined) {
        uint4 a[4], b[4], c[4];
        load_block(a, row, 0);
        if (nblocks > 1) load_block(b, row, 1);
        for (int blk = 0; blk < nblocks; blk += 3) {
            if (blk + 2 < nblocks) load_block(c, row, blk + 2);
            block_code8_ip<kForm>(x + 64 * blk, qw, T, blk, a, acc, ip, la0, la1);
            if (blk + 1 >= nblocks) break;
            if (blk + 3 < nblocks) load_block(a, row, blk + 3);
            block_code8_ip<kForm>(x + 64 * (blk + 1), qw, T, blk + 1, b, acc, ip, la0, la1);
            if (blk + 2 >= nblocks) break;
            if (blk + 4 < nblocks) load_block(b, row, blk + 4);
            block_code8_ip<kForm>(x + 64 * (blk + 2), qw, T, blk + 2, c, acc, ip, la0, la1);
        }
    } else {
        for (int blk = 0; blk < nblocks; ++blk) {
            uint4 v[4];
            load_block(v, row, blk);
            block_code8_ip<kForm>(x + 64 * blk, qw, T, blk, v, acc, ip, la0, la1);
        }
    }
    if (kForm == kRefineFullCode) return __fadd_rn(__double2float_rn(acc), kb);
    // ip1 exactly as the scan forms it; 128 * ip1 is exact
    const float ip1 = kForm == kRefineSplitInt ? __fmul_rn(width, static_cast<float>(ip))
                                               : __fadd_rn(la0, la1);
    return __fadd_rn(__fadd_rn(__fmul_rn(128.0f, ip1), __double2float_rn(acc)), kb);
}

// One CTA per query, one thread per candidate: a candidate's refine row (its 8-bit codes, D
// bytes, 32-byte sectors used whole) and its meta word are loaded before its fp64 chain.
// mode 0 refines the vanguard seeds [0, cnt) and records the seed count; mode 1 refines the
// main candidates [seed_cnt, cnt). Dynamic shared memory (refine_smem): the query as D
// doubles, its qint as D / 4 words of signed bytes, its LUT tables as 4 D floats, nprobe
// ProbeInfo.
__host__ __device__ __forceinline__ size_t refine_smem(int D, int nprobe) {
    return (size_t)D * 8 + (size_t)D + (size_t)D * 16 + (size_t)nprobe * sizeof(ProbeInfo);
}
// kLongRows: D > 128 (the rows' blocks are loaded two ahead, see refine_row_term).
template <bool kLongRows>
__global__ void __launch_bounds__(kRefineThreads) refine_kernel(IndexView ix, SearchView sv,
                                                                int mode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double *x = reinterpret_cast<double *>(smem_raw);
    uint32_t *qw = reinterpret_cast<uint32_t *>(x + ix.D);
    float *T = reinterpret_cast<float *>(qw + ix.D / 4);
    ProbeInfo *pinfo = reinterpret_cast<ProbeInfo *>(T + 4 * ix.D);
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
    const bool exact = ix.exact_base != nullptr;
    // x: the rotated query (ex-code estimate), or the raw query (exact refinement)
    if (exact) {
        for (int j = threadIdx.x; j < ix.dim; j += blockDim.x)
            x[j] = static_cast<double>(sv.raw_q[(size_t)q * ix.dim + j]);
    } else {
        for (int j = threadIdx.x; j < ix.D; j += blockDim.x)
            x[j] = static_cast<double>(sv.qr[(size_t)q * ix.D + j]);
        // the LUT estimator's tables, widened to fp32
        if (sv.lut_mode)
            for (int i = threadIdx.x; i < 4 * ix.D; i += blockDim.x)
                T[i] = __half2float(sv.lut[(size_t)q * 4 * ix.D + i]);
        // qint of dims 4t .. 4t + 3 from the query's two's-complement bit-planes (plane b,
        // word j / 32, bit 31 - j % 32 holds bit b of qint_j & 0xFF): byte i of word t
        const int W4 = 4 * ix.G16;
        const uint32_t *pl = sv.planes + (size_t)q * 8 * W4;
        for (int t = threadIdx.x; t < ix.D / 4; t += blockDim.x) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int j = 4 * t + i;
                uint32_t byte = 0;
#pragma unroll
                for (int b = 0; b < 8; ++b) byte |= ((pl[b * W4 + j / 32] >> (31 - j % 32)) & 1u) << b;
                word |= byte << (8 * i);
            }
            qw[t] = word;
        }
    }
    const int np = mode == 0 ? sv.veff : sv.nprobe;
    for (int r = threadIdx.x; r < np; r += blockDim.x) {
        const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
        pinfo[r] = ProbeInfo{ix.cl_start[c], ix.cl_size[c], sv.probe_ga[(size_t)q * sv.nprobe + r]};
    }
    __syncthreads();
    const float kb = sv.scal[q].kb, width = sv.scal[q].width;
    const int form = sv.refine_full_code ? kRefineFullCode
                                         : (sv.lut_mode ? kRefineSplitLut : kRefineSplitInt);
    const int nblocks = ix.D / 64;
    const int row4 = ix.D / 16;  // uint4 per refine row
    for (uint32_t i = from + threadIdx.x; i < to; i += blockDim.x) {
        const uint64_t rec = sv.cand_rec[(size_t)q * sv.cap + i];
        const uint32_t gid = static_cast<uint32_t>(rec & 0xFFFFFFFFu);
        const uint32_t pr = static_cast<uint32_t>(rec >> 32);
        // a record outside its probe's cluster is reported, never dereferenced
        if (pr >= static_cast<uint32_t>(np) || gid - pinfo[pr].start >= pinfo[pr].size) {
            atomicOr(sv.err, kDevBadInput);
            sv.cand_key[(size_t)q * sv.cap + i] = kKeyMax;
            continue;
        }
        const ProbeInfo p = pinfo[pr];
        const uint4 mt = __ldg(ix.meta + gid);  // {f_add_ex, f_rescale_ex, id, 0}
        if (exact) {
            // exact squared L2 distance to the base row, the fp64 fma chain over the raw
            // dimensions ascending, rounded once (cpu_refinement.cpp:168-181); a vector whose
            // row is missing is dropped (its key never ranks or sets a threshold)
            uint64_t key = kKeyMax;
            if (__ldg(ix.exact_ok + gid)) {
                const float *b = ix.exact_base + (size_t)gid * ix.dim;
                double acc = 0.0;
                for (int j0 = 0; j0 < ix.dim; j0 += 8) {
                    float bv[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) bv[u] = j0 + u < ix.dim ? __ldg(b + j0 + u) : 0.0f;
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        if (j0 + u < ix.dim) {
                            const double d = __dsub_rn(x[j0 + u], static_cast<double>(bv[u]));
                            acc = __fma_rn(d, d, acc);
                        }
                    }
                }
                key = make_key(__double2float_rn(acc), mt.z);
            }
            sv.cand_key[(size_t)q * sv.cap + i] = key;
            continue;
        }
        const uint4 *row = ix.rows + (size_t)gid * row4;
        const float2 f = make_float2(__uint_as_float(mt.x), __uint_as_float(mt.y));
        const uint32_t id = mt.z;
        float t;  // the factor of f_rescale_ex
        if (form == kRefineSplitInt)
            t = refine_row_term<kRefineSplitInt, kLongRows>(row, nblocks, x, qw, T, width, kb);
        else if (form == kRefineSplitLut)
            t = refine_row_term<kRefineSplitLut, kLongRows>(row, nblocks, x, qw, T, width, kb);
        else
            t = refine_row_term<kRefineFullCode, kLongRows>(row, nblocks, x, qw, T, width, kb);
        const float ex_d = __fadd_rn(__fadd_rn(f.x, p.g), __fmul_rn(f.y, t));
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
// With `list`, the CTAs serve the queries list[1 .. list[0]] (grid-stride) that
// topk_warp_kernel handed over.
__device__ void threshold_block(int q, const SearchView &sv, uint64_t *__restrict__ keys_out,
                                uint64_t *s_keys, int *scratch);
__global__ void __launch_bounds__(256) threshold_kernel(SearchView sv,
                                                        uint64_t *__restrict__ keys_out,
                                                        const uint32_t *__restrict__ list) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    if (!list) {
        threshold_block(blockIdx.x, sv, keys_out, s_keys, scratch);
        return;
    }
    for (uint32_t j = blockIdx.x; j < list[0]; j += gridDim.x) {
        threshold_block(static_cast<int>(list[1 + j]), sv, keys_out, s_keys, scratch);
        __syncthreads();
    }
}
__device__ void threshold_block(int q, const SearchView &sv, uint64_t *__restrict__ keys_out,
                                uint64_t *s_keys, int *scratch) {
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
// With `list`, as threshold_kernel; stats == nullptr skips the count (already added).
__device__ void merge_block(int q, const SearchView &sv, float *__restrict__ out_d,
                            uint32_t *__restrict__ out_i, unsigned long long *__restrict__ stats,
                            uint64_t *__restrict__ keys_out, uint64_t *s_keys, int *scratch);
__global__ void __launch_bounds__(256) merge_kernel(SearchView sv, float *__restrict__ out_d,
                                                    uint32_t *__restrict__ out_i,
                                                    unsigned long long *__restrict__ stats,
                                                    uint64_t *__restrict__ keys_out,
                                                    const uint32_t *__restrict__ list) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    if (!list) {
        merge_block(blockIdx.x, sv, out_d, out_i, stats, keys_out, s_keys, scratch);
        return;
    }
    for (uint32_t j = blockIdx.x; j < list[0]; j += gridDim.x) {
        merge_block(static_cast<int>(list[1 + j]), sv, out_d, out_i, stats, keys_out, s_keys,
                    scratch);
        __syncthreads();
    }
}
__device__ void merge_block(int q, const SearchView &sv, float *__restrict__ out_d,
                            uint32_t *__restrict__ out_i, unsigned long long *__restrict__ stats,
                            uint64_t *__restrict__ keys_out, uint64_t *s_keys, int *scratch) {
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
    if (threadIdx.x == 0 && stats) atomicAdd(stats, static_cast<unsigned long long>(cnt));
}

// ---- warp-level threshold (mode 0) and merge (mode 1) for k <= 32 ----------------------
// One warp per query (8 per CTA). The k-th smallest of the 32 lane minima bounds the k-th
// smallest key from above, so the k smallest keys are among those at or below it (normally
// a few dozen), which are collected and sorted. A query whose collection exceeds
// kWarpTopBuf is queued in fallback[1..] (count in fallback[0]) for the block kernel.
constexpr int kWarpTopBuf = 256;
__global__ void __launch_bounds__(256) topk_warp_kernel(SearchView sv, int mode,
                                                        float *__restrict__ out_d,
                                                        uint32_t *__restrict__ out_i,
                                                        unsigned long long *__restrict__ stats,
                                                        uint64_t *__restrict__ keys_out,
                                                        uint32_t *__restrict__ fallback) {
    __shared__ uint64_t buf[8][kWarpTopBuf];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int q = blockIdx.x * 8 + w;
    if (mode == 1 && threadIdx.x == 0) {  // candidates submitted: one atomic per CTA
        unsigned long long sum = 0;
        for (int j = blockIdx.x * 8; j < min(sv.nq, blockIdx.x * 8 + 8); ++j) sum += sv.cand_cnt[j];
        atomicAdd(stats, sum);
    }
    if (q >= sv.nq) return;  // whole warp
    const float T0 = sv.T0[q];
    const uint32_t cnt = sv.cand_cnt[q];
    const uint32_t n = mode == 0 ? sv.seed_cnt[q] : min(cnt, static_cast<uint32_t>(sv.cap));
    const uint64_t *keys = sv.cand_key + (size_t)q * sv.cap;
    const int k = sv.k;
    auto key_at = [&](uint32_t i) -> uint64_t {
        const uint64_t key = keys[i];
        return unord_f32(static_cast<uint32_t>(key >> 32)) < T0 ? key : kKeyMax;
    };
    uint64_t mn = kKeyMax;
    for (uint32_t i = lane; i < n; i += 32) {
        const uint64_t key = key_at(i);
        mn = key < mn ? key : mn;
    }
    const uint64_t tau = __shfl_sync(0xffffffffu, warp_sort_lane_keys(mn, lane), k - 1);
    uint64_t *b = buf[w];
    uint32_t m = 0;
    for (uint32_t base = 0; base < n; base += 32) {
        const uint32_t i = base + lane;
        const uint64_t key = i < n ? key_at(i) : kKeyMax;
        const bool take = key != kKeyMax && key <= tau;
        const uint32_t mask = __ballot_sync(0xffffffffu, take);
        const uint32_t pos = m + __popc(mask & ((1u << lane) - 1u));
        if (take && pos < static_cast<uint32_t>(kWarpTopBuf)) b[pos] = key;
        m += __popc(mask);
    }
    if (m > static_cast<uint32_t>(sv.topk_warp_limit)) {
        if (lane == 0) fallback[1 + atomicAdd(fallback, 1u)] = static_cast<uint32_t>(q);
        return;
    }
    int sort_n = 32;
    while (sort_n < static_cast<int>(m)) sort_n <<= 1;
    for (int i = m + lane; i < sort_n; i += 32) b[i] = kKeyMax;
    __syncwarp();
    warp_sort_smem(b, sort_n, lane);
    const uint64_t kth = b[k - 1];
    if (keys_out) {
        for (int j = lane; j < k; j += 32) keys_out[(size_t)q * k + j] = b[j];
        if (mode == 1 && q == 0 && lane == 0)
            keys_out[(size_t)sv.nq * k] = static_cast<uint32_t>(*sv.err);
    } else if (mode == 0) {
        if (lane == 0) sv.T1[q] = threshold_from_kth(kth, T0);
    } else {
        for (int j = lane; j < k; j += 32) {
            const uint64_t key = b[j];
            const bool ok = key != kKeyMax;
            out_d[(size_t)q * k + j] = ok ? unord_f32(static_cast<uint32_t>(key >> 32)) : FLT_MAX;
            out_i[(size_t)q * k + j] = ok ? static_cast<uint32_t>(key & 0xFFFFFFFFu) : 0u;
        }
        if (lane == 0)
            sv.Tcap[q] = kth != kKeyMax ? unord_f32(static_cast<uint32_t>(kth >> 32)) : T0;
    }
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
