// Query preparation and exact probe selection.
//
//  rotate_prep_kernel          q' = q * P, sumq / k1 / kb, 8-bit symmetric query bit-planes
//                              (reference: src/search/hybrid.cu:436-458,
//                               src/search/query_kernels.cuh:73-94,117-189)
//  lut_build_kernel            fp16 lookup tables of the LUT estimator (reference:
//                              src/search/query_kernels.cuh:199-221)
//  guarded_select_warp_kernel  top-nprobe by (g_add, cluster id) from the tensor-core
//  guarded_select_kernel       approximate distances (kernels_probe.cuh) plus an exact fp64
//                              recompute of the error band (reference: g_add of
//                              hybrid.cu:465-477 / query_kernels.cuh:10-64, selected by
//                              raft::matrix::select_k, hybrid.cu:485-493)
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace cora {

// queries per CTA of rotate_prep_kernel: kRotQueriesWide when D <= 128 (two groups of
// kRotQueries share the CTA's 256 threads), else kRotQueries
constexpr int kRotQueries = 8;
constexpr int kRotQueriesWide = 16;

struct QueryScalars {  // per query, 16 bytes
    float width, k1, kb, sumq;
};

// The pruning test (range_at_least, kernels_scan.cuh) needs, per query, a bound M on the
// magnitude of the scan's fl(ip1 + k1) over every possible 1-bit code. Integer estimator:
// fl(fl(width * ip) + k1) is monotone in ip, so M is taken at the ends of the reachable
// ip_int range [neg, pos] (the sums of the negative and of the positive qint).
__device__ __forceinline__ float ip_term_bound(int pos, int neg, float width, float k1) {
    const float hi = __fadd_rn(__fadd_rn(__fmul_rn(width, (float)pos), 0.0f), k1);
    const float lo = __fadd_rn(__fadd_rn(__fmul_rn(width, (float)neg), 0.0f), k1);
    return fmaxf(fabsf(hi), fabsf(lo));
}

// One CTA handles kQ queries, in kQ / 8 groups of 8 that split the CTA's threads. Each output
// dim j of q' is an fp64 chain over the input dims in ascending order (fp32 x fp32 products
// are exact in fp64, so the fused multiply-add rounds exactly like the oracle's add); the
// queries are widened to fp64 once in shared memory and the rotator is held in fp64.
// Warp w then prepares queries w, w + 8, ... Dynamic shared memory: kQ * (2 dim + D) floats.
template <int kQ>
__global__ void __launch_bounds__(256) rotate_prep_kernel(
    const float *__restrict__ raw_q, int nq, int dim, int D, int W4,
    const double *__restrict__ rotator, float c_b, float *__restrict__ qr_out,
    QueryScalars *__restrict__ scal_out, uint32_t *__restrict__ planes_out,
    float *__restrict__ qnorm2_out, float *__restrict__ ipm_out) {
    constexpr int kGroups = kQ / kRotQueries;
    extern __shared__ double smem_d[];
    double *sq = smem_d;                                        // [kQ][dim]
    float *sr = reinterpret_cast<float *>(smem_d + kQ * dim);   // [kQ][D]
    const int q0 = blockIdx.x * kQ;
    const int nqb = min(kQ, nq - q0);
    for (int i = threadIdx.x; i < kQ * dim; i += blockDim.x) {
        const int qq = i / dim;
        sq[i] = qq < nqb ? (double)raw_q[(size_t)(q0 + qq) * dim + (i - qq * dim)] : 0.0;
    }
    __syncthreads();
    constexpr int kTpg = 256 / kGroups;  // threads per group
    const int grp = threadIdx.x / kTpg;
    const double *sqg = sq + grp * kRotQueries * dim;
    // D > 128 (kQ == kRotQueries): a thread carries output dims j, j + kTpg and j + 2 kTpg
    // together (one pass over D = 768), so each query value read from shared memory feeds
    // three chains (the loads, not the fp64 FMAs, bound this loop: 1.13 ms with two columns
    // and two passes for 10K queries at D = 768, LSU pipe 52%); the D <= 128 form has one
    // column per thread anyway, and more registers would only cost it occupancy.
    constexpr int kCols = kQ == kRotQueries ? 3 : 1;
    constexpr int kRows = kCols > 1 ? 4 : 8;  // rotator rows loaded ahead of their use
    for (int j = threadIdx.x % kTpg; j < D; j += kCols * kTpg) {
        double acc[kCols][kRotQueries];
#pragma unroll
        for (int cc = 0; cc < kCols; ++cc)
#pragma unroll
            for (int qq = 0; qq < kRotQueries; ++qq) acc[cc][qq] = 0.0;
        // dim % kRows == 0 is not assumed: the tail rows read as 0 and are not accumulated
        for (int i0 = 0; i0 < dim; i0 += kRows) {
            double p[kCols][kRows];
#pragma unroll
            for (int cc = 0; cc < kCols; ++cc) {
                const int jc = j + cc * kTpg;
#pragma unroll
                for (int u = 0; u < kRows; ++u)
                    p[cc][u] = jc < D && i0 + u < dim ? __ldg(rotator + (size_t)(i0 + u) * D + jc)
                                                      : 0.0;
            }
#pragma unroll
            for (int u = 0; u < kRows; ++u) {
                if (i0 + u < dim) {
#pragma unroll
                    for (int qq = 0; qq < kRotQueries; ++qq) {
                        const double xv = sqg[qq * dim + i0 + u];
#pragma unroll
                        for (int cc = 0; cc < kCols; ++cc)
                            acc[cc][qq] = __fma_rn(xv, p[cc][u], acc[cc][qq]);
                    }
                }
            }
        }
#pragma unroll
        for (int cc = 0; cc < kCols; ++cc) {
            const int jc = j + cc * kTpg;
            if (jc >= D) continue;
#pragma unroll
            for (int qq = 0; qq < kRotQueries; ++qq) {
                const int qa = grp * kRotQueries + qq;
                const float v = (float)acc[cc][qq];
                sr[qa * D + jc] = v;
                if (qa < nqb) qr_out[(size_t)(q0 + qa) * D + jc] = v;
            }
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int qw = warp; qw < nqb; qw += 8) {
        const int q = q0 + qw;
        const float *x = sr + qw * D;
        // sumq: lane-strided fp64 partial sums, xor butterfly (identical on every lane)
        double part = 0.0;
        float amax = 0.0f;
        for (int j = lane; j < D; j += 32) {
            part = __dadd_rn(part, (double)x[j]);
            amax = fmaxf(amax, fabsf(x[j]));
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            part = __dadd_rn(part, __shfl_xor_sync(0xffffffffu, part, off));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        }
        const float sf = (float)part;
        const float width = fmaxf(__fdiv_rn(amax, 127.0f), 1e-30f);
        const float inv = __fdiv_rn(1.0f, width);
        // ||q'||^2 for the approximate coarse distances (any order: it only feeds the filter)
        double nrm = 0.0;
        for (int j = lane; j < D; j += 32) nrm = __fma_rn((double)x[j], (double)x[j], nrm);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) nrm += __shfl_xor_sync(0xffffffffu, nrm, off);
        if (lane == 0) {
            QueryScalars s;
            s.width = width;
            s.k1 = __fmul_rn(sf, -0.5f);
            s.kb = __fmul_rn(sf, c_b);
            s.sumq = sf;
            scal_out[q] = s;
            qnorm2_out[q] = (float)nrm;
        }
        uint32_t *pl = planes_out + (size_t)q * 8 * W4;
        int pos = 0, neg = 0;  // sums of the positive and of the negative qint
        for (int w = 0; w < W4; ++w) {
            const int j = w * 32 + lane;
            int v = 0;
            if (j < D) {
                v = __float2int_rn(__fmul_rn(x[j], inv));
                v = max(-128, min(127, v));
            }
            pos += max(v, 0);
            neg += min(v, 0);
            const uint32_t bits = static_cast<uint32_t>(v) & 0xFFu;
#pragma unroll
            for (int b = 0; b < 8; ++b) {
                const uint32_t m = __brev(__ballot_sync(0xffffffffu, (bits >> b) & 1u));
                if (lane == 0) pl[b * W4 + w] = m;
            }
        }
        // [neg, pos] is the range of sum_i b_i qint_i over every 1-bit code (the scan's bound)
        pos = __reduce_add_sync(0xffffffffu, pos);
        neg = __reduce_add_sync(0xffffffffu, neg);
        if (ipm_out && lane == 0) ipm_out[q] = ip_term_bound(pos, neg, width, __fmul_rn(sf, -0.5f));
    }
}

// ---- LUT estimator tables -----------------------------------------------------------
// The reference's default estimator (KernelType::Lut4Bit) forms ip1 = <q', b> from fp16
// tables: entry (g, p) of nibble group g (dims 4g .. 4g + 3) and 4-bit pattern p (bit 3 =
// dim 4g, ..., bit 0 = dim 4g + 3) is half(s), s the fp32 sum, starting from 0, of the
// selected q' in dimension order (query_kernels.cuh:199-221). Tables are stored as
// lut[q][g][p], 16 halves (32 bytes) per group. One warp per query, 8 queries per CTA.
//
// The bound M of the pruning test: the exact sum of a code's entries lies in [Lo, Hi], Lo / Hi
// the sums over the groups of their smallest / largest entry (sums of halves, exact in
// fp64). ip1 = acc0 + acc1 sums at most D / 8 entries per accumulator in fp32, so it is
// within ((D / 8) + 1) 2^-24 A <= 2^-16 A of the exact sum (A = sum_g max_p |entry(g, p)|,
// D <= 1024), and fl(ip1 + k1) is then within
// M = (max(|Hi + k1|, |Lo + k1|) + 2^-16 A) (1 + 2^-22) of zero (every step rounded upwards).
constexpr int kLutWarps = 8;
__global__ void __launch_bounds__(32 * kLutWarps) lut_build_kernel(
    const float *__restrict__ qr, const QueryScalars *__restrict__ scal, int nq, int D,
    __half *__restrict__ lut, float *__restrict__ ipm) {
    const int lane = threadIdx.x & 31;
    const int q = blockIdx.x * kLutWarps + (threadIdx.x >> 5);
    if (q >= nq) return;  // whole warp
    const float4 *x4 = reinterpret_cast<const float4 *>(qr + (size_t)q * D);
    double A = 0.0, Hi = 0.0, Lo = 0.0;  // sums of halves: exact in fp64
    for (int g = lane; g < D / 4; g += 32) {
        const float4 v = __ldg(x4 + g);
        __align__(16) __half h[16];
        double hmax = 0.0, hmin = 0.0;  // p = 0 gives 0
#pragma unroll
        for (int p = 0; p < 16; ++p) {
            float sum = 0.0f;
            if (p & 8) sum = __fadd_rn(sum, v.x);
            if (p & 4) sum = __fadd_rn(sum, v.y);
            if (p & 2) sum = __fadd_rn(sum, v.z);
            if (p & 1) sum = __fadd_rn(sum, v.w);
            h[p] = __float2half_rn(sum);
            const double e = (double)__half2float(h[p]);
            hmax = fmax(hmax, e);
            hmin = fmin(hmin, e);
        }
        uint4 *dst = reinterpret_cast<uint4 *>(lut + ((size_t)q * (D / 4) + g) * 16);
        dst[0] = *reinterpret_cast<const uint4 *>(h);
        dst[1] = *reinterpret_cast<const uint4 *>(h + 8);
        A += fmax(hmax, -hmin);
        Hi += hmax;
        Lo += hmin;
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        A += __shfl_xor_sync(0xffffffffu, A, off);
        Hi += __shfl_xor_sync(0xffffffffu, Hi, off);
        Lo += __shfl_xor_sync(0xffffffffu, Lo, off);
    }
    if (lane == 0) {
        // max |t| over t in [Lo + k1, Hi + k1] is max(Hi + k1, -(Lo + k1)), each bounded
        // outwards (k1 may carry bits below the halves' 2^-24 grid)
        const double k1 = (double)scal[q].k1;
        const double span = fmax(__dadd_ru(Hi, k1), -__dadd_rd(Lo, k1));
        const double m = __dmul_ru(__dadd_ru(span, __dmul_ru(A, 0x1p-16)), 1.0 + 0x1p-22);
        ipm[q] = __double2float_ru(m);
    }
}

// Exact coarse distance of the search contract: g(q, c) = fp32( sum_j fma(d_j, d_j) ) with
// d_j = q'_j - c_j in fp64, ascending j (reference: hybrid.cu:465-477 forms the same
// ||q'||^2 + ||c||^2 - 2 q'.c in fp32).
// The centroid row is loaded 32 dims at a time (eight 16-byte loads in flight; rows are
// 16-byte aligned since D % 64 == 0) ahead of the chain, which stays in ascending order.
__device__ __forceinline__ float exact_centroid_dist(const float *__restrict__ x,
                                                     const float *__restrict__ c, int D) {
    double acc = 0.0;
    const float4 *c4 = reinterpret_cast<const float4 *>(c);
    for (int j0 = 0; j0 < D; j0 += 32) {
        float4 v[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) v[t] = __ldg(c4 + j0 / 4 + t);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float cv[4] = {v[t].x, v[t].y, v[t].z, v[t].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const double d = __dsub_rn((double)x[j0 + 4 * t + u], (double)cv[u]);
                acc = __fma_rn(d, d, acc);
            }
        }
    }
    return (float)acc;
}

// The approximate distances come from probe_gemm_kernel (tensor cores, kernels_probe.cuh),
// with |approx - g| <= kApproxEpsTF32 * (||q'|| + max ||c||)^2.

// One CTA per query: the nprobe probes of the contract (smallest exact g, ties by cluster
// id) from approximate distances. tau = nprobe-th smallest approx; every exact top-nprobe
// centroid has approx <= tau + 2E (E the approx error bound), so only those candidates are
// recomputed exactly (fp64) and selected. More candidates than the shared buffer holds (a
// pathological tie band) fall back to exact distances for every centroid of the query,
// written over its approximate row. Dynamic shared memory: see guarded_select_smem().
// list == nullptr: query blockIdx.x; otherwise the queries list[1 .. list[0]] (grid-stride),
// the ones guarded_select_warp_kernel handed over.
__device__ void guarded_select_block(int q, float *__restrict__ approx,
                                     const float *__restrict__ chunk_min, int nlist, size_t ld,
                                     int nprobe, int cand_cap, const float *__restrict__ qr,
                                     const float *__restrict__ qnorm2,
                                     const float *__restrict__ cent, float cmax, int D, double eps,
                                     int *__restrict__ probe_ids, float *__restrict__ probe_g);

__global__ void __launch_bounds__(256) guarded_select_kernel(
    float *__restrict__ approx, const float *__restrict__ chunk_min, int nlist, size_t ld,
    int nprobe, int cand_cap, const float *__restrict__ qr, const float *__restrict__ qnorm2,
    const float *__restrict__ cent, float cmax, int D, double eps, int *__restrict__ probe_ids,
    float *__restrict__ probe_g, const uint32_t *__restrict__ list) {
    if (!list) {
        guarded_select_block(blockIdx.x, approx, chunk_min, nlist, ld, nprobe, cand_cap, qr,
                             qnorm2, cent, cmax, D, eps, probe_ids, probe_g);
        return;
    }
    const uint32_t n = list[0];
    for (uint32_t j = blockIdx.x; j < n; j += gridDim.x) {
        guarded_select_block(static_cast<int>(list[1 + j]), approx, chunk_min, nlist, ld, nprobe,
                             cand_cap, qr, qnorm2, cent, cmax, D, eps, probe_ids, probe_g);
        __syncthreads();  // shared memory is reused by the next query
    }
}

// chunk_min (nullable): the probe GEMM's per-chunk row minima. With them, and at least nprobe
// chunks, the upper bound of tau comes from a selection over the chunk minima (nlist / 32
// keys) instead of the whole row, and the band is collected from the chunks whose minimum
// lies inside it.
__device__ void guarded_select_block(int q, float *__restrict__ approx,
                                     const float *__restrict__ chunk_min, int nlist, size_t ld,
                                     int nprobe, int cand_cap, const float *__restrict__ qr,
                                     const float *__restrict__ qnorm2,
                                     const float *__restrict__ cent, float cmax, int D, double eps,
                                     int *__restrict__ probe_ids, float *__restrict__ probe_g) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int S2 = next_pow2(nprobe);
    uint64_t *sel = reinterpret_cast<uint64_t *>(smem_raw);          // S2
    uint64_t *ckeys = sel + S2;                                       // cand_cap
    uint32_t *cidx = reinterpret_cast<uint32_t *>(ckeys + cand_cap);  // cand_cap
    float *x = reinterpret_cast<float *>(cidx + cand_cap);            // D
    __shared__ int scratch[256 + 3];
    __shared__ int s_ncand;
    float *row = approx + (size_t)q * ld;  // ld: row stride (nlist rounded up to 4 floats)
    for (int j = threadIdx.x; j < D; j += blockDim.x) x[j] = qr[(size_t)q * D + j];
    if (threadIdx.x == 0) s_ncand = 0;
    auto approx_key = [&](uint32_t c) -> uint64_t { return make_key(row[c], c); };
    const int nchunk = (nlist + 31) / 32;
    const float *cm = chunk_min ? chunk_min + (size_t)q * chunk_stride(nlist) : nullptr;
    if (cm && nchunk >= nprobe) {
        // the nprobe-th smallest chunk minimum bounds tau from above (nprobe distinct chunks
        // hold a centroid at or below it)
        auto chunk_key = [&](uint32_t j) -> uint64_t { return make_key(__ldg(cm + j), j); };
        block_select_smallest(chunk_key, static_cast<uint32_t>(nchunk), nprobe, sel, scratch);
    } else {
        block_select_smallest(approx_key, static_cast<uint32_t>(nlist), nprobe, sel, scratch);
    }
    const double tau = (double)unord_f32(static_cast<uint32_t>(sel[nprobe - 1] >> 32));
    const double r = sqrt((double)qnorm2[q]) + (double)cmax;
    const double bound = tau + 2.0 * (eps * r * r + 1e-30);
    for (int c = threadIdx.x; c < nlist; c += blockDim.x) {
        if ((!cm || (double)__ldg(cm + (c >> 5)) <= bound) && (double)row[c] <= bound) {
            const int pos = atomicAdd(&s_ncand, 1);
            if (pos < cand_cap) cidx[pos] = static_cast<uint32_t>(c);
        }
    }
    __syncthreads();
    const int ncand = s_ncand;
    if (ncand <= cand_cap) {
        for (int i = threadIdx.x; i < ncand; i += blockDim.x) {
            const uint32_t c = cidx[i];
            ckeys[i] = make_key(exact_centroid_dist(x, cent + (size_t)c * D, D), c);
        }
        __syncthreads();
        auto exact_key = [&](uint32_t i) -> uint64_t { return ckeys[i]; };
        block_select_smallest(exact_key, static_cast<uint32_t>(ncand), nprobe, sel, scratch);
    } else {
        for (int c = threadIdx.x; c < nlist; c += blockDim.x)
            row[c] = exact_centroid_dist(x, cent + (size_t)c * D, D);
        __syncthreads();
        block_select_smallest(approx_key, static_cast<uint32_t>(nlist), nprobe, sel, scratch);
    }
    for (int rr = threadIdx.x; rr < nprobe; rr += blockDim.x) {
        const uint64_t key = sel[rr];
        probe_ids[(size_t)q * nprobe + rr] = static_cast<int>(key & 0xFFFFFFFFu);
        probe_g[(size_t)q * nprobe + rr] = unord_f32(static_cast<uint32_t>(key >> 32));
    }
}

__host__ __device__ inline size_t guarded_select_smem(int nprobe, int cand_cap, int D) {
    return (size_t)next_pow2(nprobe) * 8 + (size_t)cand_cap * 12 + (size_t)D * 4;
}

// One warp per query (8 per CTA), nprobe <= 32: the same selection without block-wide radix
// passes. The nprobe-th smallest chunk minimum, tau_ub, is >= tau (nprobe values lie at or
// below it), so {approx <= tau_ub + 2E} contains the guard band {approx <= tau + 2E},
// and recomputing that superset exactly selects the same probes (a centroid outside the band
// can never beat one of the true top-nprobe). It is normally a few dozen centroids; a query
// whose set exceeds kGuardWarpBand is queued in fallback[1..] (count in fallback[0]) for
// guarded_select_kernel. Dynamic shared memory: guarded_select_warp_smem(D).
constexpr int kGuardWarpBand = 256;
constexpr int kGuardWarps = 8;
__host__ __device__ inline size_t guarded_select_warp_slice(int D) {
    return (size_t)D * 4 + (size_t)kGuardWarpBand * 12;
}
__host__ __device__ inline size_t guarded_select_warp_smem(int D) {
    return kGuardWarps * guarded_select_warp_slice(D);
}

//
// The bound and the band come from the per-chunk minima the probe GEMM writes
// (chunk_min[q * chunk_stride(nlist) + j] = min of row q's columns 32j .. 32j + 31): lane l's
// group is its chunks l, l + 32, ..., and only the chunks whose minimum is inside the band
// are read from the distance row (128 coalesced bytes each), so a row is not read in full.
// The nprobe-th smallest of a row's nchunk <= 32 R chunk minima (cm), by an exact radix
// selection over their order keys held in registers (R per lane, padding: the largest key),
// one bit per warp-wide count.
template <int R>
__device__ __forceinline__ float radix_tau_regs(const float *__restrict__ cm, int nchunk,
                                                int nprobe, int lane) {
    uint32_t kr[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int c = lane + 32 * i;
        kr[i] = c < nchunk ? ord_f32(__ldg(cm + c)) : 0xFFFFFFFFu;
    }
    uint32_t prefix = 0, remaining = static_cast<uint32_t>(nprobe);
    for (int bit = 31; bit >= 0; --bit) {
        const uint32_t above = bit == 31 ? 0u : ~((2u << bit) - 1u);  // bits above `bit`
        uint32_t cnt = 0;
#pragma unroll
        for (int i = 0; i < R; ++i)
            cnt += ((kr[i] & above) == prefix && !((kr[i] >> bit) & 1u)) ? 1u : 0u;
        cnt = __reduce_add_sync(0xffffffffu, cnt);
        if (cnt < remaining) {
            remaining -= cnt;
            prefix |= 1u << bit;
        }
    }
    return unord_f32(prefix);
}

__global__ void __launch_bounds__(256) guarded_select_warp_kernel(
    const float *__restrict__ approx, const float *__restrict__ chunk_min, int nlist, size_t ld,
    int nq, int nprobe, const float *__restrict__ qr, const float *__restrict__ qnorm2,
    const float *__restrict__ cent, float cmax, int D, double eps, int *__restrict__ probe_ids,
    float *__restrict__ probe_g, uint32_t *__restrict__ fallback) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q = blockIdx.x * kGuardWarps + w;
    if (q >= nq) return;  // whole warp
    float *x = reinterpret_cast<float *>(smem_raw + w * guarded_select_warp_slice(D));
    uint64_t *keys = reinterpret_cast<uint64_t *>(x + D);  // D % 64 == 0: 8-byte aligned
    uint32_t *cidx = reinterpret_cast<uint32_t *>(keys + kGuardWarpBand);
    const float *row = approx + (size_t)q * ld;
    const int nchunk = (nlist + 31) / 32;
    const float *cm = chunk_min + (size_t)q * chunk_stride(nlist);
    for (int j = lane; j < D; j += 32) x[j] = qr[(size_t)q * D + j];

    // tau_ub: the nprobe-th smallest chunk minimum (nprobe distinct chunks each hold a
    // centroid at or below it, so it bounds the nprobe-th smallest approximate distance from
    // above, and is that distance itself when the nprobe nearest lie in distinct chunks).
    // Rows of at most 32 chunks: one chunk per lane, sorted; longer rows: an exact radix
    // selection over the chunk minima's order keys, one bit per warp-wide count (the keys
    // in registers up to 1024 chunks, nlist <= 32768).
    double tau_ub;
    if (nchunk <= 32) {
        const float mn = lane < nchunk ? __ldg(cm + lane) : FLT_MAX;
        const uint64_t kth = __shfl_sync(0xffffffffu,
                                         warp_sort_lane_keys(make_key(mn, lane), lane), nprobe - 1);
        tau_ub = (double)unord_f32(static_cast<uint32_t>(kth >> 32));
    } else if (nchunk <= 128) {
        tau_ub = (double)radix_tau_regs<4>(cm, nchunk, nprobe, lane);
    } else if (nchunk <= 256) {
        tau_ub = (double)radix_tau_regs<8>(cm, nchunk, nprobe, lane);
    } else if (nchunk <= 512) {
        tau_ub = (double)radix_tau_regs<16>(cm, nchunk, nprobe, lane);
    } else if (nchunk <= 1024) {
        tau_ub = (double)radix_tau_regs<32>(cm, nchunk, nprobe, lane);
    } else {
        uint32_t prefix = 0, remaining = static_cast<uint32_t>(nprobe);
        for (int bit = 31; bit >= 0; --bit) {
            const uint32_t above = bit == 31 ? 0u : ~((2u << bit) - 1u);  // bits above `bit`
            uint32_t cnt = 0;
            for (int c = lane; c < nchunk; c += 32) {
                const uint32_t key = ord_f32(__ldg(cm + c));
                cnt += ((key & above) == prefix && !((key >> bit) & 1u)) ? 1u : 0u;
            }
            cnt = __reduce_add_sync(0xffffffffu, cnt);
            if (cnt < remaining) {
                remaining -= cnt;
                prefix |= 1u << bit;
            }
        }
        tau_ub = (double)unord_f32(prefix);
    }
    const double r = sqrt((double)qnorm2[q]) + (double)cmax;
    const double bound = tau_ub + 2.0 * (eps * r * r + 1e-30);

    uint32_t cnt = 0;
    for (int cb = 0; cb < nchunk; cb += 32) {
        const int c = cb + lane;
        uint32_t chunks = __ballot_sync(0xffffffffu, c < nchunk && (double)__ldg(cm + c) <= bound);
        while (chunks) {  // warp-uniform: the chunks that can hold a band member, 4 at a time
            int col[4];
            float v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {  // every load first: one round trip per 4 chunks
                col[u] = chunks ? 32 * (cb + __ffs(chunks) - 1) + lane : nlist;
                chunks &= chunks - 1;
                v[u] = col[u] < nlist ? __ldg(row + col[u]) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const bool take = col[u] < nlist && (double)v[u] <= bound;
                const uint32_t m = __ballot_sync(0xffffffffu, take);
                const uint32_t pos = cnt + __popc(m & ((1u << lane) - 1u));
                if (take && pos < kGuardWarpBand) cidx[pos] = static_cast<uint32_t>(col[u]);
                cnt += __popc(m);
            }
        }
    }
    if (cnt > kGuardWarpBand) {
        if (lane == 0) fallback[1 + atomicAdd(fallback, 1u)] = static_cast<uint32_t>(q);
        return;
    }
    __syncwarp();
    for (uint32_t i = lane; i < cnt; i += 32) {
        const uint32_t c = cidx[i];
        keys[i] = make_key(exact_centroid_dist(x, cent + (size_t)c * D, D), c);
    }
    __syncwarp();
    if (cnt <= 32) {
        const uint64_t key = warp_sort_lane_keys(lane < (int)cnt ? keys[lane] : kKeyMax, lane);
        if (lane < nprobe) {
            probe_ids[(size_t)q * nprobe + lane] = static_cast<int>(key & 0xFFFFFFFFu);
            probe_g[(size_t)q * nprobe + lane] = unord_f32(static_cast<uint32_t>(key >> 32));
        }
    } else {
        const int n2 = next_pow2(static_cast<int>(cnt));
        for (int i = static_cast<int>(cnt) + lane; i < n2; i += 32) keys[i] = kKeyMax;
        __syncwarp();
        warp_sort_smem(keys, n2, lane);
        for (int j = lane; j < nprobe; j += 32) {
            const uint64_t key = keys[j];
            probe_ids[(size_t)q * nprobe + j] = static_cast<int>(key & 0xFFFFFFFFu);
            probe_g[(size_t)q * nprobe + j] = unord_f32(static_cast<uint32_t>(key >> 32));
        }
    }
}
// Inner-product metric: the estimator's additive term of every (query, probe) pair,
// g_add = -<q', c'> (index/query.hpp:99-108; the reference CPU path probes by L2 distance and
// takes the dot product with the probed centroid, ivf/ivf.hpp:681-706), as the fp32 rounding
// of the fp64 fma chain over the dimensions in ascending order. One warp per query, one
// lane per probe.
__global__ void __launch_bounds__(256) ip_gadd_kernel(const float *__restrict__ qr,
                                                      const float *__restrict__ cent,
                                                      const int *__restrict__ probe_ids, int nq,
                                                      int nprobe, int D,
                                                      float *__restrict__ probe_ga) {
    const int lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (q >= nq) return;
    const float *x = qr + (size_t)q * D;
    for (int r = lane; r < nprobe; r += 32) {
        const float4 *c4 = reinterpret_cast<const float4 *>(
            cent + (size_t)probe_ids[(size_t)q * nprobe + r] * D);
        double acc = 0.0;
        for (int j0 = 0; j0 < D; j0 += 4) {
            const float4 c = __ldg(c4 + j0 / 4);
            acc = __fma_rn((double)x[j0], (double)c.x, acc);
            acc = __fma_rn((double)x[j0 + 1], (double)c.y, acc);
            acc = __fma_rn((double)x[j0 + 2], (double)c.z, acc);
            acc = __fma_rn((double)x[j0 + 3], (double)c.w, acc);
        }
        probe_ga[(size_t)q * nprobe + r] = -__double2float_rn(acc);
    }
}

__host__ __device__ inline int guarded_select_cap(int nprobe) {
    const int c = 2 * nprobe > 1024 ? 2 * nprobe : 1024;
    return c < 8192 ? c : 8192;
}

}  // namespace cora
