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
// threads per query (one CTA) of the refine kernels; measured on config 2 with one thread
// per candidate: 64 -> 0.202 ms, 128 -> 0.192, 256 -> 0.188 (seed refine 0.080 / 0.072 /
// 0.075)
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

// Summation order of the refinement's fp64 inner products (the kernels below and the oracle
// form them identically): a refine row is read as 16-byte chunks, chunk c = dimensions
// 16c .. 16c + 15. Partial sum j (j = 0 .. 7) runs over the chunks c with c % 8 == j, chunks
// ascending and dimensions ascending within a chunk, one fma per dimension (every product
// x_d * c_d is exact in fp64); the eight partials are combined as
// ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)) and the sum is rounded once to fp32.
// Partials without chunks (D < 128) stay +0.
constexpr int kRefinePartials = 8;
// Shared-memory stride of a chunk's 16 query doubles: 2 doubles of padding put the chunks
// that the lanes of a row read at once (128 bytes apart otherwise: one bank) into distinct
// banks.
constexpr int kXChunk = 18;
// Chunks a lane loads per round with one lane per row (4 or 8).
#ifndef CORA_REFINE_ROW_CHUNKS
#define CORA_REFINE_ROW_CHUNKS 4
#endif
constexpr int kRefineRowChunks = CORA_REFINE_ROW_CHUNKS;

// One chunk of a refine row (v: the 8-bit codes c = 128 b + u of dims 16c .. 16c + 15, 4 per
// word, dimension order) against the rotated query (xc = x + 16 c, fp64 in shared memory),
// continuing partial sum `acc`. Each byte becomes the double c (or u = c & 127) exactly as
// (2^52 + c) - 2^52 from its bit pattern.
//   kRefineSplitInt: acc accumulates <x, u>, and ip accumulates sum_i b_i qint_i with dp4a
//     over the code words' top bits and the query's qint bytes (qv: qint of the chunk's dims,
//     4 per word as signed bytes), exact in int32;
//   kRefineSplitLut: acc accumulates <x, u> (the LUT sums are formed separately);
//   kRefineFullCode: acc accumulates <x, 128 b + u>.
template <int kForm>
__device__ __forceinline__ void chunk_code8_ip(const double *__restrict__ xc, const uint4 qv,
                                               const uint4 v, double &acc, int &ip) {
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    const uint32_t q4[4] = {qv.x, qv.y, qv.z, qv.w};
    const double2 *x2 = reinterpret_cast<const double2 *>(xc);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
        const uint32_t w = kForm == kRefineFullCode ? w4[h] : (w4[h] & 0x7F7F7F7Fu);
        if (kForm == kRefineSplitInt)
            ip = __dp4a(static_cast<int>((w4[h] >> 7) & 0x01010101u), static_cast<int>(q4[h]), ip);
        const double2 xa = x2[2 * h], xb = x2[2 * h + 1];
        const double xs[4] = {xa.x, xa.y, xb.x, xb.y};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t c = __byte_perm(w, 0u, 0x4440u | i);
            const double cd = __dsub_rn(__hiloint2double(0x43300000, static_cast<int>(c)),
                                        4503599627370496.0);
            acc = __fma_rn(xs[i], cd, acc);
        }
    }
}

// The LUT estimator's nibble patterns of a chunk's four 4-dimension groups, group k at bits
// 4k .. 4k + 3: the group's code bits b (the bytes' top bits), its first dimension at bit 3
// of the pattern (the order of ip_from_lut).
__device__ __forceinline__ uint32_t chunk_patterns(const uint4 v) {
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t out = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t w = w4[k];
        out |= (((w >> 4) & 8u) | ((w >> 13) & 4u) | ((w >> 22) & 2u) | (w >> 31)) << (4 * k);
    }
    return out;
}

// Dynamic shared memory of the refine kernels: the query as D / 16 chunks of kXChunk doubles
// (the raw query, dim <= D doubles, for the exact refinement), its qint as D / 4 words of
// signed bytes, its LUT tables as 4 D floats, nprobe ProbeInfo.
__host__ __device__ __forceinline__ size_t refine_x_doubles(int D) {
    return (size_t)(D / 16) * kXChunk;
}
__host__ __device__ __forceinline__ size_t refine_smem(int D, int nprobe) {
    return refine_x_doubles(D) * 8 + (size_t)D + (size_t)D * 16 +
           (size_t)nprobe * sizeof(ProbeInfo);
}

// Stages the refinement's per-query operands in shared memory: x (the rotated query, or the
// raw query when `exact`), the LUT tables widened to fp32 (LUT form), qint words (integer
// form), and the probes' cluster ranges and additive terms.
__device__ __forceinline__ void refine_stage(const IndexView &ix, const SearchView &sv, int q,
                                             int np, bool exact, double *x, uint32_t *qw,
                                             float *T, ProbeInfo *pinfo) {
    if (exact) {
        for (int j = threadIdx.x; j < ix.dim; j += blockDim.x)
            x[j] = static_cast<double>(sv.raw_q[(size_t)q * ix.dim + j]);
    } else {
        for (int j = threadIdx.x; j < ix.D; j += blockDim.x)
            x[(j / 16) * kXChunk + j % 16] = static_cast<double>(sv.qr[(size_t)q * ix.D + j]);
        if (sv.lut_mode && !sv.refine_full_code)
            for (int i = threadIdx.x; i < 4 * ix.D; i += blockDim.x)
                T[i] = __half2float(sv.lut[(size_t)q * 4 * ix.D + i]);
        if (!sv.lut_mode && !sv.refine_full_code) {
            // qint of dims 4t .. 4t + 3 from the query's two's-complement bit-planes (plane
            // b, word j / 32, bit 31 - j % 32 holds bit b of qint_j & 0xFF): byte i of word t
            const int W4 = 4 * ix.G16;
            const uint32_t *pl = sv.planes + (size_t)q * 8 * W4;
            for (int t = threadIdx.x; t < ix.D / 4; t += blockDim.x) {
                uint32_t word = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int j = 4 * t + i;
                    uint32_t byte = 0;
#pragma unroll
                    for (int b = 0; b < 8; ++b)
                        byte |= ((pl[b * W4 + j / 32] >> (31 - j % 32)) & 1u) << b;
                    word |= byte << (8 * i);
                }
                qw[t] = word;
            }
        }
    }
    for (int r = threadIdx.x; r < np; r += blockDim.x) {
        const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
        pinfo[r] = ProbeInfo{ix.cl_start[c], ix.cl_size[c], sv.probe_ga[(size_t)q * sv.nprobe + r]};
    }
}

// The candidate range of a refine launch: mode 0 refines the vanguard seeds [0, cnt) and
// records the seed count, mode 1 the main candidates [seed_cnt, cnt); false when empty.
__device__ __forceinline__ bool refine_range(const SearchView &sv, int q, int mode,
                                             uint32_t &from, uint32_t &to) {
    const uint32_t cnt = sv.cand_cnt[q];
    const uint32_t cap = static_cast<uint32_t>(sv.cap);
    to = min(cnt, cap);
    if (mode == 0) {
        from = 0;
        if (threadIdx.x == 0) sv.seed_cnt[q] = to;
    } else {
        from = sv.seed_cnt[q];
    }
    return from < to;
}

using RefineKernelFn = void (*)(IndexView, SearchView, int);

// One CTA per query; kLanes lanes (1, 4 or 8) take a candidate's row: lane l of a row's group
// loads and accumulates chunks l, l + kLanes, ... (kC at a time), so with 4 or 8 lanes each
// load instruction reads 16 kLanes consecutive bytes of a row, and holds partial sums
// l + kLanes t (with one lane per row: all eight, and the warp's 32 rows read the same query
// doubles at once). The partials are combined in the fixed order above by xor-shuffles
// between the row's lanes and in-lane adds (fp64 addition commutes, so every lane of the row
// ends with the same bits); the integer estimate ip_int is reduced by shuffles (exact); the
// LUT form's two fp32 chains (even groups, odd groups, ascending, as the scan forms them) run
// in the row's even and odd lanes over the chunks' patterns, gathered by shuffles (both in
// the one lane when kLanes is 1). Lane 0 writes the key.
// CTAs per SM the one-lane-per-row kernel is compiled for (48 registers, a few bytes of
// spill; measured at D = 128: candidates 0.248 -> 0.241 ms against the uncapped 64)
#ifndef CORA_REFINE_ROW_MINB
#define CORA_REFINE_ROW_MINB 10
#endif
template <int kLanes, int kC, int kForm>
__global__ void __launch_bounds__(kRefineThreads, kLanes == 1 ? CORA_REFINE_ROW_MINB : 1)
    refine_kernel(IndexView ix, SearchView sv, int mode) {
    static_assert(kLanes == 1 || kLanes == 4 || kLanes == 8, "1, 4 or 8 lanes per row");
    constexpr int P = kRefinePartials / kLanes;  // partials per lane
    // a round covers whole partial cycles, or (one lane per row, kC = 4) half of one: the
    // rounds then alternate between partials 0 .. 3 and 4 .. 7
    static_assert(kC % P == 0 || (kLanes == 1 && kC == 4), "rounds and partials");
    constexpr int kRowsPerWarp = 32 / kLanes;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double *x = reinterpret_cast<double *>(smem_raw);
    uint32_t *qw = reinterpret_cast<uint32_t *>(x + refine_x_doubles(ix.D));
    float *T = reinterpret_cast<float *>(qw + ix.D / 4);
    ProbeInfo *pinfo = reinterpret_cast<ProbeInfo *>(T + 4 * ix.D);
    const int q = blockIdx.x;
    uint32_t from, to;
    if (!refine_range(sv, q, mode, from, to)) return;  // uniform across the block
    const int np = mode == 0 ? sv.veff : sv.nprobe;
    refine_stage(ix, sv, q, np, false, x, qw, T, pinfo);
    __syncthreads();
    const float kb = sv.scal[q].kb, width = sv.scal[q].width;
    const int lane = threadIdx.x & 31, gl = lane % kLanes, gw = lane / kLanes;
    const int warp = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
    const int nl = ix.D / (16 * kLanes);  // chunks per lane (the host picks kLanes | D / 16)
    const int row4 = ix.D / 16;
    const uint4 *qw4 = reinterpret_cast<const uint4 *>(qw);
    for (uint32_t base = from + warp * kRowsPerWarp; base < to;
         base += nwarp * kRowsPerWarp) {  // warp-uniform: every lane takes the shuffles
        const uint32_t i = base + gw;
        bool ok = i < to;
        uint32_t gid = 0, pr = 0;
        if (ok) {
            const uint64_t rec = sv.cand_rec[(size_t)q * sv.cap + i];
            gid = static_cast<uint32_t>(rec & 0xFFFFFFFFu);
            pr = static_cast<uint32_t>(rec >> 32);
            // a record outside its probe's cluster is reported, never dereferenced
            if (pr >= static_cast<uint32_t>(np) || gid - pinfo[pr].start >= pinfo[pr].size) {
                if (gl == 0) {
                    atomicOr(sv.err, kDevBadInput);
                    sv.cand_key[(size_t)q * sv.cap + i] = kKeyMax;
                }
                ok = false;
            }
        }
        uint4 mt = make_uint4(0u, 0u, 0u, 0u);
        if (ok && gl == 0) mt = __ldg(ix.meta + gid);  // {f_add_ex, f_rescale_ex, id, 0}
        const uint4 *row = ix.rows + (size_t)gid * row4 + gl;
        double acc[P];
#pragma unroll
        for (int t = 0; t < P; ++t) acc[t] = 0.0;
        int ip = 0;
        float la = 0.0f;   // LUT form: even lanes the even groups' chain, odd lanes the odd one
        float la1 = 0.0f;  // (one lane per row: la the even chain, la1 the odd one)
        for (int s0 = 0; s0 < nl; s0 += kC) {
            uint4 v[kC];
#pragma unroll
            for (int u = 0; u < kC; ++u)
                v[u] = (ok && s0 + u < nl) ? __ldg(row + kLanes * (s0 + u))
                                           : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int u = 0; u < kC; ++u) {
                if (s0 + u < nl) {
                    const int c = gl + kLanes * (s0 + u);
                    const uint4 qv = kForm == kRefineSplitInt ? qw4[c] : make_uint4(0u, 0u, 0u, 0u);
                    if constexpr (kC % P == 0) {
                        chunk_code8_ip<kForm>(x + kXChunk * c, qv, v[u], acc[u % P], ip);
                    } else {
                        if (s0 & 4)
                            chunk_code8_ip<kForm>(x + kXChunk * c, qv, v[u], acc[4 + u], ip);
                        else
                            chunk_code8_ip<kForm>(x + kXChunk * c, qv, v[u], acc[u], ip);
                    }
                }
            }
            if (kForm == kRefineSplitLut) {
                uint32_t pats[kC];
#pragma unroll
                for (int u = 0; u < kC; ++u) pats[u] = chunk_patterns(v[u]);
                const int par = gl & 1;
#pragma unroll
                for (int u = 0; u < kC; ++u) {
                    if (s0 + u < nl) {  // uniform
#pragma unroll
                        for (int l = 0; l < kLanes; ++l) {
                            const uint32_t m =
                                kLanes == 1 ? pats[u] : __shfl_sync(0xffffffffu, pats[u], l, kLanes);
                            const int c = l + kLanes * (s0 + u);
                            if (kLanes == 1) {
#pragma unroll
                                for (int k = 0; k < 4; ++k) {
                                    const float e = T[(4 * c + k) * 16 + ((m >> (4 * k)) & 15u)];
                                    if (k & 1)
                                        la1 = __fadd_rn(la1, e);
                                    else
                                        la = __fadd_rn(la, e);
                                }
                            } else {
#pragma unroll
                                for (int k2 = 0; k2 < 2; ++k2) {
                                    const int k = 2 * k2 + par;
                                    la = __fadd_rn(la, T[(4 * c + k) * 16 + ((m >> (4 * k)) & 15u)]);
                                }
                            }
                        }
                    }
                }
            }
        }
        // combine the partials: ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7))
#pragma unroll
        for (int b = 1; b < kRefinePartials; b <<= 1) {
            if (b < kLanes) {
#pragma unroll
                for (int t = 0; t < P; ++t)
                    acc[t] = __dadd_rn(acc[t], __shfl_xor_sync(0xffffffffu, acc[t], b));
            } else {
                const int tb = b / kLanes;
#pragma unroll
                for (int t = 0; t < P; t += 2 * tb) acc[t] = __dadd_rn(acc[t], acc[t + tb]);
            }
        }
        float ip1 = 0.0f;
        if (kForm == kRefineSplitInt) {
#pragma unroll
            for (int b = 1; b < kLanes; b <<= 1) ip += __shfl_xor_sync(0xffffffffu, ip, b);
            ip1 = __fmul_rn(width, static_cast<float>(ip));  // as the scan forms it
        } else if (kForm == kRefineSplitLut) {
            if (kLanes == 1)
                ip1 = __fadd_rn(la, la1);
            else
                ip1 = __fadd_rn(__shfl_sync(0xffffffffu, la, 0, kLanes),
                                __shfl_sync(0xffffffffu, la, 1, kLanes));
        }
        if (ok && gl == 0) {
            float t;  // the factor of f_rescale_ex; 128 * ip1 is exact
            if (kForm == kRefineFullCode)
                t = __fadd_rn(__double2float_rn(acc[0]), kb);
            else
                t = __fadd_rn(__fadd_rn(__fmul_rn(128.0f, ip1), __double2float_rn(acc[0])), kb);
            const float ex_d = __fadd_rn(__fadd_rn(__uint_as_float(mt.x), pinfo[pr].g),
                                         __fmul_rn(__uint_as_float(mt.y), t));
            sv.cand_key[(size_t)q * sv.cap + i] = make_key(ex_d, mt.z);
        }
    }
}

// Exact refinement (--exact-base): one CTA per query, one thread per candidate, the exact
// squared L2 distance to the candidate's fp32 base row as an fp64 fma chain over the raw
// dimensions ascending, rounded once (cpu_refinement.cpp:168-181); a vector whose row is
// missing is dropped (its key never ranks or sets a threshold). Modes as refine_kernel.
__global__ void __launch_bounds__(kRefineThreads) refine_exact_kernel(IndexView ix,
                                                                      SearchView sv, int mode) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    double *x = reinterpret_cast<double *>(smem_raw);
    uint32_t *qw = reinterpret_cast<uint32_t *>(x + refine_x_doubles(ix.D));
    float *T = reinterpret_cast<float *>(qw + ix.D / 4);
    ProbeInfo *pinfo = reinterpret_cast<ProbeInfo *>(T + 4 * ix.D);
    const int q = blockIdx.x;
    uint32_t from, to;
    if (!refine_range(sv, q, mode, from, to)) return;  // uniform across the block
    const int np = mode == 0 ? sv.veff : sv.nprobe;
    refine_stage(ix, sv, q, np, true, x, qw, T, pinfo);
    __syncthreads();
    for (uint32_t i = from + threadIdx.x; i < to; i += blockDim.x) {
        const uint64_t rec = sv.cand_rec[(size_t)q * sv.cap + i];
        const uint32_t gid = static_cast<uint32_t>(rec & 0xFFFFFFFFu);
        const uint32_t pr = static_cast<uint32_t>(rec >> 32);
        if (pr >= static_cast<uint32_t>(np) || gid - pinfo[pr].start >= pinfo[pr].size) {
            atomicOr(sv.err, kDevBadInput);
            sv.cand_key[(size_t)q * sv.cap + i] = kKeyMax;
            continue;
        }
        uint64_t key = kKeyMax;
        if (__ldg(ix.exact_ok + gid)) {
            const uint32_t id = __ldg(ix.meta + gid).z;
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
            key = make_key(__double2float_rn(acc), id);
        }
        sv.cand_key[(size_t)q * sv.cap + i] = key;
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

// Probe exchange (probing split by query over the shards): shard r probes queries
// [r s, min(nq, (r + 1) s)), s = ceil(nq / world), and sends one word per (query, probe rank)
// of its slice, (bits of g << 32) | cluster, then its device error word.
__global__ void __launch_bounds__(256) pack_probes_kernel(const int *__restrict__ probe_ids,
                                                          const float *__restrict__ probe_g,
                                                          size_t n, const int *__restrict__ err,
                                                          uint64_t *__restrict__ out,
                                                          size_t stride) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        out[i] = (static_cast<uint64_t>(__float_as_uint(probe_g[i])) << 32) |
                 static_cast<uint32_t>(probe_ids[i]);
    if (blockIdx.x == 0 && threadIdx.x == 0) out[stride - 1] = static_cast<uint32_t>(*err);
}

// Every shard's slice back into the probe lists of the whole batch (nq x np), and every
// shard's error word ORed into this shard's.
__global__ void __launch_bounds__(256) unpack_probes_kernel(const uint64_t *__restrict__ recv,
                                                            int world, size_t stride, size_t slice,
                                                            size_t nq, int np,
                                                            int *__restrict__ probe_ids,
                                                            float *__restrict__ probe_g,
                                                            int *__restrict__ err) {
    const size_t n = nq * np;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
        const size_t q = i / np, r = q / slice;
        const uint64_t w = recv[r * stride + (q - r * slice) * np + (i - q * np)];
        probe_ids[i] = static_cast<int>(static_cast<uint32_t>(w));
        probe_g[i] = __uint_as_float(static_cast<uint32_t>(w >> 32));
    }
    if (blockIdx.x == 0 && threadIdx.x < world) {
        const int e = static_cast<int>(recv[threadIdx.x * stride + stride - 1]);
        if (e) atomicOr(err, e);
    }
}

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
