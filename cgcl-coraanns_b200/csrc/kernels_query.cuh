// Query preparation and coarse probing kernels.
//
//  rotate_prep_kernel   q' = q * P, sumq / k1 / kb, 8-bit symmetric query bit-planes
//                       (reference: src/search/hybrid.cu:436-458,
//                        src/search/query_kernels.cuh:73-94,117-189)
//  centroid_dist_kernel g_add(q, c) = ||q' - c'||^2 for every (query, centroid)
//                       (reference: hybrid.cu:465-477, query_kernels.cuh:10-64)
//  select_probes_kernel top-nprobe by (g_add, cluster id)
//                       (reference: raft::matrix::select_k, hybrid.cu:485-493)
#pragma once
#include "common.cuh"

namespace cora {

constexpr int kRotQueries = 8;  // queries per CTA in rotate_prep_kernel

struct QueryScalars {  // per query, 16 bytes
    float width, k1, kb, sumq;
};

// One CTA handles kRotQueries queries. Each output dim j of q' is an fp64 chain over the
// input dims in ascending order (fp32 x fp32 products are exact in fp64, so the fused
// multiply-add rounds exactly like the oracle's add). Warp w then prepares query w.
// Dynamic shared memory: kRotQueries * (dim + D) floats.
__global__ void __launch_bounds__(256) rotate_prep_kernel(
    const float *__restrict__ raw_q, int nq, int dim, int D, int W4,
    const float *__restrict__ rotator, float c_b, float *__restrict__ qr_out,
    QueryScalars *__restrict__ scal_out, uint32_t *__restrict__ planes_out) {
    extern __shared__ float smem_f[];
    float *sq = smem_f;                       // [kRotQueries][dim]
    float *sr = smem_f + kRotQueries * dim;   // [kRotQueries][D]
    const int q0 = blockIdx.x * kRotQueries;
    const int nqb = min(kRotQueries, nq - q0);
    for (int i = threadIdx.x; i < kRotQueries * dim; i += blockDim.x) {
        const int qq = i / dim;
        sq[i] = qq < nqb ? raw_q[(size_t)(q0 + qq) * dim + (i - qq * dim)] : 0.0f;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < D; j += blockDim.x) {
        double acc[kRotQueries];
#pragma unroll
        for (int qq = 0; qq < kRotQueries; ++qq) acc[qq] = 0.0;
        for (int i = 0; i < dim; ++i) {
            const double p = (double)__ldg(rotator + (size_t)i * D + j);
#pragma unroll
            for (int qq = 0; qq < kRotQueries; ++qq)
                acc[qq] = __fma_rn((double)sq[qq * dim + i], p, acc[qq]);
        }
#pragma unroll
        for (int qq = 0; qq < kRotQueries; ++qq) {
            const float v = (float)acc[qq];
            sr[qq * D + j] = v;
            if (qq < nqb) qr_out[(size_t)(q0 + qq) * D + j] = v;
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp >= nqb) return;
    const int q = q0 + warp;
    const float *x = sr + warp * D;
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
    if (lane == 0) {
        QueryScalars s;
        s.width = width;
        s.k1 = __fmul_rn(sf, -0.5f);
        s.kb = __fmul_rn(sf, c_b);
        s.sumq = sf;
        scal_out[q] = s;
    }
    uint32_t *pl = planes_out + (size_t)q * 8 * W4;
    for (int w = 0; w < W4; ++w) {
        const int j = w * 32 + lane;
        int v = 0;
        if (j < D) {
            v = __float2int_rn(__fmul_rn(x[j], inv));
            v = max(-128, min(127, v));
        }
        const uint32_t bits = static_cast<uint32_t>(v) & 0xFFu;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const uint32_t m = __brev(__ballot_sync(0xffffffffu, (bits >> b) & 1u));
            if (lane == 0) pl[b * W4 + w] = m;
        }
    }
}

// Exact coarse distances: g[q][c] = fp32( sum_j fma((q'_j - c_j), (q'_j - c_j)) ) in fp64,
// ascending j. 64 x 64 output tile per CTA, 256 threads with 4 x 4 outputs each.
constexpr int kDistTile = 64, kDistK = 32;
__global__ void __launch_bounds__(256) centroid_dist_kernel(
    const float *__restrict__ qr, int nq, const float *__restrict__ cent, int nlist, int D,
    float *__restrict__ g_out) {
    __shared__ float sq[kDistK][kDistTile + 1];
    __shared__ float sc[kDistK][kDistTile + 1];
    const int qbase = blockIdx.y * kDistTile, cbase = blockIdx.x * kDistTile;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    double acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.0;
    for (int k0 = 0; k0 < D; k0 += kDistK) {
        for (int i = threadIdx.x; i < kDistK * kDistTile; i += blockDim.x) {
            const int row = i / kDistK, kk = i % kDistK;
            const int qi = qbase + row, ci = cbase + row;
            sq[kk][row] = qi < nq ? qr[(size_t)qi * D + k0 + kk] : 0.0f;
            sc[kk][row] = ci < nlist ? cent[(size_t)ci * D + k0 + kk] : 0.0f;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < kDistK; ++kk) {
            double qv[4], cv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) qv[a] = (double)sq[kk][ty * 4 + a];
#pragma unroll
            for (int b = 0; b < 4; ++b) cv[b] = (double)sc[kk][tx * 4 + b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const double d = __dsub_rn(qv[a], cv[b]);
                    acc[a][b] = __fma_rn(d, d, acc[a][b]);
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int qi = qbase + ty * 4 + a;
        if (qi >= nq) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int ci = cbase + tx * 4 + b;
            if (ci < nlist) g_out[(size_t)qi * nlist + ci] = (float)acc[a][b];
        }
    }
}

// One CTA per query: the nprobe smallest (g, c) keys, ascending, by block radix selection
// over the query's row of distances. Dynamic shared memory: next_pow2(nprobe) keys.
__global__ void __launch_bounds__(256) select_probes_kernel(const float *__restrict__ g,
                                                            int nlist, int nprobe,
                                                            int *__restrict__ probe_ids,
                                                            float *__restrict__ probe_g) {
    extern __shared__ uint64_t smem_k[];
    __shared__ int scratch[256 + 3];
    const int q = blockIdx.x;
    const float *row = g + (size_t)q * nlist;
    auto key_at = [&](uint32_t c) -> uint64_t { return make_key(row[c], c); };
    block_select_smallest(key_at, static_cast<uint32_t>(nlist), nprobe, smem_k, scratch);
    for (int r = threadIdx.x; r < nprobe; r += blockDim.x) {
        const uint64_t key = smem_k[r];
        probe_ids[(size_t)q * nprobe + r] = static_cast<int>(key & 0xFFFFFFFFu);
        probe_g[(size_t)q * nprobe + r] = unord_f32(static_cast<uint32_t>(key >> 32));
    }
}

}  // namespace cora
