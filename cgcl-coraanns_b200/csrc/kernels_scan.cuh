// 1-bit RaBitQ estimator scan: per-cluster query grouping, vanguard seeding and the main
// pruned scan.
//
// Device scan layout ("scan planes"): for cluster c with start s_c (its first vector's
// position in the reference's cluster order) and size n_c, uint4 entry
//   scan4[(G16 + 1) * s_c + g * n_c + i]
// holds, for g < G16, 1-bit code words 4g..4g+3 of vector i (word w covers dims 32w..32w+31
// with dim 32w+b at bit 31-b, as src/index/search_data.cpp:71), and for g == G16 the
// factors {f_add, f_rescale, f_error, 0}. Each plane of a cluster is contiguous, so a tile
// of TV vectors is G16 + 1 TMA bulk copies of TV * 16 bytes.
//
// Estimator (reference src/search/filter_kernels.cuh:79-114, 693-696):
//   ip_int = sum_{j<7} popc(x & plane_j) << j  -  popc(x & plane_7) << 7      (exact)
//          = sum_i b_i qint_i, evaluated as byte dot products (dp4a) for D <= 128 and as
//            bit-plane popcounts above (both exact in int32)
//   ip1    = width * ip_int
//   low    = (f_add + g_add) + f_rescale * (ip1 + k1) - f_error * sqrt(max(g, 0))
// with g the squared L2 distance to the probed centroid and g_add = g (L2) or -<q', c'>
// (inner product; the reference CPU path's set_g_add, index/query.hpp:99-108 and
// ivf/ivf.hpp:699-706); or, with the LUT estimator (the reference's default kernel type, filter_kernels.cuh:
// 283-306, 655-696), ip1 = acc0 + acc1 from the query's fp16 tables (lut_build_kernel):
// nibble n of code word w (bits 31 - 4n .. 28 - 4n, dims 32w + 4n ..) looks up entry
// (8w + n, nibble) and is added, in fp32 and in order, to acc0 for even n, acc1 for odd n.
//
// Search phases (all on one stream):
//  1. vanguard pairs (probe rank r < veff) are grouped by cluster and scanned once; their
//     lower bounds are stored in an HBM buffer (`lows`, 4 B per (pair, vector));
//  2. per vanguard pair, the best `keep` keys (low, gid) among low < T0 become seeds;
//  3. after the seeds are refined, T1 = min(T0, k-th smallest seed distance);
//  4. the remaining pairs (r >= veff) are grouped by cluster and scanned against T1, and the
//     stored lows of the vanguard pairs are filtered against T1 (skipping their seeds).
// When the lows buffer would not fit its budget, step 1-2 run as one kernel per vanguard
// pair instead (vanguard_rescan_kernel) and step 4 rescans the vanguard clusters. Step 4
// leaves out every (pair, cluster), (pair, item) and (pair, 32-vector chunk) whose factor
// range proves all its lows >= T1 (range_at_least): the candidate set is unchanged.
#pragma once
#include "common.cuh"
#include "kernels_query.cuh"

namespace cora {

constexpr int kScanThreads = 256;
constexpr int kMaxPairsPerItem = 32;

// Vectors each scan_kernel thread evaluates per pass over an item's pairs (D <= 128 only):
// the query words read from shared memory then serve that many vectors.
#ifndef CORA_SCAN_VPT
#define CORA_SCAN_VPT 1
#endif

template <int G16>
struct ScanShape {
    static constexpr int TV = 256;                     // vectors per staged tile (rescan)
    // LUT estimator: floats per pair of the tables staged in shared memory (32 G16 nibble
    // groups x 16; groups past D / 4 hold zeros, which leave the sums unchanged) and the
    // pairs per grouped item that keep them within the shared-memory budget
    static constexpr int kLutFloats = 512 * G16;
    static constexpr int kLutPairs = G16 == 1 ? 32 : (G16 == 2 ? 16 : 8);
    // tiles in flight in scan_kernel (its shared memory: kStages x kStageEntries x 16 B);
    // deep enough to hide the TMA latency when an item serves few queries
    static constexpr int kStages = G16 <= 2 ? 4 : 2;
    static constexpr int W4 = 4 * G16;                 // 32-bit code words per vector
    static constexpr int kStageEntries = (G16 + 1) * TV;
    // scan_kernel's tiles: kScanThreads x VPT vectors
    static constexpr int VPT = G16 == 1 ? CORA_SCAN_VPT : 1;
    static constexpr int kScanTV = 256 * VPT;
    static constexpr int kScanStageEntries = (G16 + 1) * kScanTV;
};

struct ScanItem {
    uint32_t cluster, pair_begin, pair_count, pad;
};

struct IndexView {
    const uint4 *scan4;          // scan planes
    const uint32_t *cl_start;    // nlist
    const uint32_t *cl_size;     // nlist
    // factor ranges (FactorRange) of every 32-vector chunk of every cluster (cluster c's
    // chunk j at cl_chunk[c] + j) and of whole clusters (cl_range[c]); see chunk_ranges_kernel
    const float4 *chunk_range;
    const uint32_t *cl_chunk;    // nlist + 1
    const float4 *cl_range;      // nlist
    // refine rows (build_refine_rows_kernel): per vector its D 8-bit codes c = 128 b + u
    // (b the 1-bit code, u the 7-bit ex code), one byte per dimension
    const uint4 *rows;           // N x D / 16
    const uint4 *meta;           // N: {f_add_ex, f_rescale_ex, id, 0}
    // exact FP32 refinement (nullptr: off): base row of every vector (N x dim, its original
    // id's row of the caller's base) and whether that row exists (N)
    const float *exact_base;
    const uint8_t *exact_ok;
    int nlist, D, G16, LC, dim;
};

struct SearchView {
    int nq, k, nprobe, veff, keep, cap;
    const float *raw_q;          // nq x dim, the search's input queries (exact refinement)
    const QueryScalars *scal;    // nq
    const float *ipm;            // nq: bound on |fl(ip1 + k1)| (ip_term_bound / lut_build_kernel)
    const uint32_t *planes;      // nq x 8 x W4
    const __half *lut;           // nq x (D / 4) x 16: LUT estimator tables (lut_mode only)
    int lut_mode;                // 1: the scan's ip1 comes from the LUT estimator
    const float *qr;             // nq x D
    const int *probe_ids;        // nq x nprobe
    const float *probe_g;        // nq x nprobe: squared L2 distance to the probed centroid
    // nq x nprobe: the estimator's additive query term g_add (L2: probe_g itself; inner
    // product: -<q', c'>); its error term is always sqrt(probe_g)
    const float *probe_ga;
    const float *T0;             // nq, seeded thresholds (never modified by a search)
    float *Tcap;                 // nq, thresholds after the search (capture_thresholds)
    float *T1;                   // nq
    uint64_t *bound;             // nq x veff
    uint32_t *cand_cnt;          // nq
    uint32_t *seed_cnt;          // nq
    uint64_t *cand_rec;          // nq x cap : gid | (probe rank << 32)
    uint64_t *cand_key;          // nq x cap : ord(ex) << 32 | id
    float *lows;                 // vanguard lower bounds (lows mode), see vg_off
    uint64_t *vg_off;            // nq x veff: each vanguard pair's slice offset in lows
    uint64_t lows_cap;           // capacity of lows (floats)
    unsigned long long *lows_top;  // bump allocator of lows slices (zeroed per search)
    int *err;
    int warp_select_limit;       // keys a warp may collect before queueing a block selection
    int topk_warp_limit;         // the same for the threshold / final top-k (topk_warp_kernel)
    int refine_full_code;        // refine with <q', 128 b + u> instead of 128 ip1 + ip2
};

// ---- factor ranges and the lower-bound test that skips whole chunks -------------------
// A factor range {min f_add, max |f_add|, max |f_rescale|, max |f_error|} over a set of
// vectors bounds every lower bound the scan computes for them against one pair:
//   low = fl(fl(fl(f_add + g) + fl(f_rescale * t)) - fl(f_error * gerr)),  |t| <= M,
// where t = fl(fl(width * ip) + k1) is monotone in ip, so M (its largest magnitude over the
// reachable ip in [neg, pos]) is taken at an end of that range. Each of the five roundings
// errs by at most 2^-24 of a magnitude below S = max|f_add| + |g| + max|f_rescale| M +
// max|f_error| gerr, so low >= L - 2^-20 S with L = min f_add + g - max|f_rescale| M -
// max|f_error| gerr. When that is >= T, no vector of the set has low < T: skipping it
// leaves the candidate set unchanged. NaN factors fall out of the min/max (fminf/fmaxf
// ignore NaN) and their lows (NaN) are never below T either.
__device__ __forceinline__ bool range_at_least(float4 fr, float g, float M, float gerr,
                                               float T) {
    const double r = (double)fr.z * M, e = (double)fr.w * gerr;
    const double L = ((double)fr.x + g) - r - e;
    const double S = (double)fr.y + fabs((double)g) + r + e;
    return L - 0x1p-20 * S >= (double)T;
}

// Pair pruning of the main pass's grouping (cl_range == nullptr: none): a (query, probe)
// pair is left out when its cluster's factor range proves every low >= T1 of the query, the
// test scan_kernel also applies per item and per chunk.
struct PairPrune {
    const float4 *cl_range;      // nlist
    const float *probe_g;        // nq x nprobe (error term)
    const float *probe_ga;       // nq x nprobe (additive term)
    const float *ipm;            // nq
    const float *T1;             // nq
};
__device__ __forceinline__ bool pair_pruned(const PairPrune &pp, int q, int r, int c,
                                            int nprobe) {
    if (!pp.cl_range) return false;
    const size_t at = (size_t)q * nprobe + r;
    return range_at_least(pp.cl_range[c], pp.probe_ga[at], pp.ipm[q],
                          __fsqrt_rn(fmaxf(pp.probe_g[at], 0.0f)), pp.T1[q]);
}

// ---- per-cluster query grouping (CSR of (query, probe rank) pairs by cluster) --------
// Pairs with probe rank in [r_lo, r_hi) whose cluster is owned by this shard (owned ==
// nullptr: all) and that pair_pruned keeps are grouped; a pair is packed as (q << 16) | r.
__global__ void count_pairs_kernel(const int *__restrict__ probe_ids, int nq, int nprobe,
                                   int r_lo, int r_hi, const uint8_t *__restrict__ owned,
                                   PairPrune pp, uint32_t *__restrict__ cnt) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)nq * nprobe) return;
    const int r = static_cast<int>(i % nprobe);
    if (r < r_lo || r >= r_hi) return;
    const int c = probe_ids[i];
    if (owned && !owned[c]) return;
    if (pair_pruned(pp, static_cast<int>(i / nprobe), r, c, nprobe)) return;
    atomicAdd(cnt + c, 1u);
}

// Single-CTA exclusive scan of pair counts into offsets and of per-cluster item counts
// (ceil(count / ppi), ppi = pairs per item <= kMaxPairsPerItem) into item offsets; the item
// total lands in *n_items.
__global__ void __launch_bounds__(1024) scan_pairs_kernel(const uint32_t *__restrict__ cnt,
                                                          int nlist, int ppi,
                                                          uint32_t *__restrict__ off,
                                                          uint32_t *__restrict__ item_off,
                                                          uint32_t *__restrict__ n_items) {
    __shared__ uint32_t s_pairs[1024], s_items[1024];
    const int t = threadIdx.x;
    const int per = (nlist + 1023) / 1024;
    const int b = t * per, e = min(nlist, b + per);
    uint32_t sp = 0, si = 0;
    for (int c = b; c < e; ++c) {
        sp += cnt[c];
        si += (cnt[c] + ppi - 1) / ppi;
    }
    s_pairs[t] = sp;
    s_items[t] = si;
    __syncthreads();
    for (int d = 1; d < 1024; d <<= 1) {
        const uint32_t vp = t >= d ? s_pairs[t - d] : 0, vi = t >= d ? s_items[t - d] : 0;
        __syncthreads();
        s_pairs[t] += vp;
        s_items[t] += vi;
        __syncthreads();
    }
    uint32_t rp = s_pairs[t] - sp, ri = s_items[t] - si;
    for (int c = b; c < e; ++c) {
        off[c] = rp;
        item_off[c] = ri;
        rp += cnt[c];
        ri += (cnt[c] + ppi - 1) / ppi;
    }
    if (t == 1023) {
        off[nlist] = s_pairs[1023];
        *n_items = s_items[1023];
    }
}

__global__ void scatter_pairs_kernel(const int *__restrict__ probe_ids, int nq, int nprobe,
                                     int r_lo, int r_hi, const uint8_t *__restrict__ owned,
                                     PairPrune pp, const uint32_t *__restrict__ off,
                                     uint32_t *__restrict__ cursor,
                                     uint32_t *__restrict__ pairs) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)nq * nprobe) return;
    const int r = static_cast<int>(i % nprobe);
    if (r < r_lo || r >= r_hi) return;
    const int c = probe_ids[i];
    if (owned && !owned[c]) return;
    const int q = static_cast<int>(i / nprobe);
    if (pair_pruned(pp, q, r, c, nprobe)) return;
    const uint32_t pos = atomicAdd(cursor + c, 1u);
    pairs[off[c] + pos] = (static_cast<uint32_t>(q) << 16) | static_cast<uint32_t>(r);
}

__global__ void emit_items_kernel(const uint32_t *__restrict__ cnt,
                                  const uint32_t *__restrict__ off,
                                  const uint32_t *__restrict__ item_off, int nlist, int ppi,
                                  ScanItem *__restrict__ items) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= nlist) return;
    const uint32_t n = cnt[c];
    const uint32_t base = item_off[c];
    const uint32_t up = static_cast<uint32_t>(ppi);
    for (uint32_t t = 0; t * up < n; ++t) {
        ScanItem it;
        it.cluster = static_cast<uint32_t>(c);
        it.pair_begin = off[c] + t * up;
        it.pair_count = min(up, n - t * up);
        it.pad = 0;
        items[base + t] = it;
    }
}

// Lows slices: each vanguard pair gets round_up(n_c, 4) floats (16-byte aligned slices, so
// the select and filter kernels read them as float4), bump-allocated per item by the lows
// pass of scan_kernel; the worst case (every query probing the largest clusters) is what
// prepare_workspace reserves.
__host__ __device__ __forceinline__ uint32_t lows_slice(uint32_t n) { return (n + 3u) & ~3u; }

// One CTA per cluster: the factor range of each 32-vector chunk (warp-wide reductions) and
// of the whole cluster. Built once when the index is loaded.
__global__ void __launch_bounds__(256) chunk_ranges_kernel(const uint4 *__restrict__ scan4,
                                                           const uint32_t *__restrict__ cl_start,
                                                           const uint32_t *__restrict__ cl_size,
                                                           const uint32_t *__restrict__ cl_chunk,
                                                           int G16, float4 *__restrict__ chunk_range,
                                                           float4 *__restrict__ cl_range) {
    __shared__ float4 s_red[8];
    const int c = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t s = cl_start[c], n = cl_size[c];
    const float inf = __int_as_float(0x7f800000);
    float4 acc = make_float4(inf, 0.0f, 0.0f, 0.0f);
    for (uint32_t k = warp; k * 32 < n; k += 8) {
        const uint32_t i = k * 32 + lane;
        float4 v = make_float4(inf, 0.0f, 0.0f, 0.0f);
        if (i < n) {
            const uint4 f = scan4[(size_t)(G16 + 1) * s + (size_t)G16 * n + i];
            const float fa = __uint_as_float(f.x);
            v = make_float4(fa, fabsf(fa), fabsf(__uint_as_float(f.y)),
                            fabsf(__uint_as_float(f.z)));
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            v.x = fminf(v.x, __shfl_xor_sync(0xffffffffu, v.x, off));
            v.y = fmaxf(v.y, __shfl_xor_sync(0xffffffffu, v.y, off));
            v.z = fmaxf(v.z, __shfl_xor_sync(0xffffffffu, v.z, off));
            v.w = fmaxf(v.w, __shfl_xor_sync(0xffffffffu, v.w, off));
        }
        if (lane == 0) chunk_range[cl_chunk[c] + k] = v;
        acc = make_float4(fminf(acc.x, v.x), fmaxf(acc.y, v.y), fmaxf(acc.z, v.z),
                          fmaxf(acc.w, v.w));
    }
    if (lane == 0) s_red[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w)
            acc = make_float4(fminf(acc.x, s_red[w].x), fmaxf(acc.y, s_red[w].y),
                              fmaxf(acc.z, s_red[w].z), fmaxf(acc.w, s_red[w].w));
        cl_range[c] = acc;
    }
}

// ---- shared pieces ------------------------------------------------------------------
template <int G16, int TVT = ScanShape<G16>::TV>
__device__ __forceinline__ void issue_tile(uint4 *stage_buf, uint64_t *bar, const uint4 *scan4,
                                           size_t cbase, int n, int v0, int tv) {
    const uint32_t bytes = static_cast<uint32_t>(tv) * 16u;
    mbar_arrive_expect_tx(bar, bytes * (G16 + 1));
#pragma unroll
    for (int g = 0; g <= G16; ++g)
        bulk_g2s(stage_buf + g * TVT, scan4 + cbase + (size_t)g * n + v0, bytes,
                 bar);
}

// ---- exact 1-bit x 8-bit inner product ---------------------------------------------
// With offset-binary query planes p'_j (bit j of qint + 128, i.e. the two's-complement
// planes with plane 7 inverted), sum_i b_i qint_i = sum_j 2^j popc(x & p'_j) - 128 popc(x),
// an integer identity, so the result equals the reference's
// sum_{j<7} popc(x & p_j) << j - popc(x & p_7) << 7 (filter_kernels.cuh:79-104) bit for
// bit. The weighted popcount sum of one 128-bit group (8 planes x 4 words) is formed by a
// carry-save adder tree over the low weights: words of equal weight are combined three at a
// time into a sum word and a carry word of twice the weight. POPC issues at a quarter of the
// logic-op rate on this SM, and a full tree (10 POPC) left the logic pipe the bottleneck, so
// the tree stops at weight 2^4 and the words of weights 2^5..2^7 (plus the carries into
// 2^5) are counted directly: 5 + 15 POPC, about 20 fewer logic ops, both pipes near balance.
__device__ __forceinline__ void full_add(uint32_t &s, uint32_t &c, uint32_t a, uint32_t b,
                                         uint32_t d) {
    s = a ^ b ^ d;
    c = (a & b) | (d & (a ^ b));
}
__device__ __forceinline__ void half_add(uint32_t &s, uint32_t &c, uint32_t a, uint32_t b) {
    s = a ^ b;
    c = a & b;
}

// Weights combined by the adder tree (2^0 .. 2^(kCsaLevels-1)); 8 = the full tree. Measured
// on config 2 with this form in both scan passes (before the byte dot products replaced it
// for D <= 128): 4 -> 1.35 ms, 5 -> 1.25, 6 -> 1.27, 7 -> 1.36, 8 -> 1.41.
#ifndef CORA_CSA_LEVELS
#define CORA_CSA_LEVELS 5
#endif
constexpr int kCsaLevels = CORA_CSA_LEVELS;
static_assert(kCsaLevels >= 2 && kCsaLevels <= 8, "adder tree depth");
// Resident CTAs per SM that scan_kernel's register budget is sized for: 4 (<= 64 registers)
// for D <= 128, where it was measured 3% faster than 2 or 3 on config 2; 2 above.
#ifndef CORA_SCAN_MINB
#define CORA_SCAN_MINB(G16) ((G16) == 1 ? 4 : 2)
#endif

// sum_j 2^j sum_t popc(x_t & p'_{j,t}) for one group; P points at the group's plane words
// (plane j at P + j * W4, 4 consecutive words).
template <int W4>
__device__ __forceinline__ int group_weighted_popc(uint4 x, const uint32_t *__restrict__ P) {
    uint32_t a[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint4 p = *reinterpret_cast<const uint4 *>(P + j * W4);
        a[j][0] = x.x & p.x;
        a[j][1] = x.y & p.y;
        a[j][2] = x.z & p.z;
        a[j][3] = x.w & p.w;
    }
    uint32_t s, t, cA, cB, cC, nA, nB, nC;
    int total;
    // weight 2^0: 4 words
    full_add(s, cA, a[0][0], a[0][1], a[0][2]);
    half_add(s, cB, s, a[0][3]);
    total = __popc(s);
    // weight 2^1: 4 words + 2 carries
    full_add(s, nA, a[1][0], a[1][1], a[1][2]);
    full_add(t, nB, a[1][3], cA, cB);
    half_add(s, nC, s, t);
    total += __popc(s) << 1;
    cA = nA;
    cB = nB;
    cC = nC;
    // weights 2^2 .. 2^(L-1): 4 words + 3 carries each
#pragma unroll
    for (int j = 2; j < kCsaLevels; ++j) {
        full_add(s, nA, a[j][0], a[j][1], a[j][2]);
        full_add(t, nB, a[j][3], cA, cB);
        full_add(s, nC, s, t, cC);
        total += __popc(s) << j;
        cA = nA;
        cB = nB;
        cC = nC;
    }
    if (kCsaLevels == 8) {  // full tree: the carries of weight 2^8 and their carry (2^9)
        full_add(s, nA, cA, cB, cC);
        return total + (__popc(s) << 8) + (__popc(nA) << 9);
    }
    // weights 2^L .. 2^7 counted directly (the 3 carries into 2^L as well)
    total += (__popc(cA) + __popc(cB) + __popc(cC)) << kCsaLevels;
#pragma unroll
    for (int j = kCsaLevels; j < 8; ++j)
        total += (__popc(a[j][0]) + __popc(a[j][1]) + __popc(a[j][2]) + __popc(a[j][3])) << j;
    return total;
}

// popc of the whole code times 128: the query-independent part of the identity.
template <int G16>
__device__ __forceinline__ int code_bias(const uint4 (&code)[G16]) {
    int px = 0;
#pragma unroll
    for (int g = 0; g < G16; ++g)
        px += __popc(code[g].x) + __popc(code[g].y) + __popc(code[g].z) + __popc(code[g].w);
    return px << 7;
}

// sum_i b_i qint_i of one code against one query's offset-binary planes; `bias` is
// code_bias(code), computed once per vector.
template <int G16>
__device__ __forceinline__ int ip_int_from_planes(const uint4 (&code)[G16],
                                                  const uint32_t *__restrict__ P, int bias) {
    constexpr int W4 = ScanShape<G16>::W4;
    int t = 0;
#pragma unroll
    for (int g = 0; g < G16; ++g) t += group_weighted_popc<W4>(code[g], P + 4 * g);
    return t - bias;
}

// ---- the same inner product through byte dot products -------------------------------
// Code word x_w (dims 32w .. 32w + 31, dim 32w + b at bit 31 - b) is split into eight words
// of 0/1 bytes, e_{w,s} = (x_w >> s) & 0x01010101: byte m is the bit of dim
// 32w + 31 - s - 8m. The query word Q_{w,s} holds qint of those four dims as signed bytes,
// so sum_{w,s} dp4a(e_{w,s}, Q_{w,s}) = sum_i b_i qint_i exactly (int32 accumulation,
// |sum| <= 128 D). The split is done once per vector and serves every query of the item.
#ifndef CORA_SCAN_DP4A
#define CORA_SCAN_DP4A 1
#endif
constexpr bool kScanDp4a = CORA_SCAN_DP4A != 0;

// Q_{w,s} of one query from its two's-complement bit-planes (plane j word w at pl[j*W4+w]):
// bit s + 8m of plane j is bit j of byte m.
__device__ __forceinline__ uint32_t query_byte_word(const uint32_t *__restrict__ pl, int w,
                                                    int s, int W4) {
    uint32_t v = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) v |= ((__ldg(pl + j * W4 + w) >> s) & 0x01010101u) << j;
    return v;
}

template <int G16>
__device__ __forceinline__ void split_code_bytes(const uint4 (&code)[G16],
                                                 uint32_t (&e)[32 * G16]) {
#pragma unroll
    for (int g = 0; g < G16; ++g) {
        const uint32_t x[4] = {code[g].x, code[g].y, code[g].z, code[g].w};
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int s = 0; s < 8; ++s) e[(4 * g + t) * 8 + s] = (x[t] >> s) & 0x01010101u;
    }
}

// sum_i b_i qint_i from the split code and one query's byte words Q (Q_{w,s} at Q[8w + s]).
template <int G16>
__device__ __forceinline__ int ip_int_from_bytes(const uint32_t (&e)[32 * G16],
                                                 const uint32_t *__restrict__ Q) {
    int acc[4] = {0, 0, 0, 0};  // four independent chains (dp4a latency)
#pragma unroll
    for (int w = 0; w < 4 * G16; ++w) {
        const uint4 a = *reinterpret_cast<const uint4 *>(Q + 8 * w);
        const uint4 b = *reinterpret_cast<const uint4 *>(Q + 8 * w + 4);
        acc[0] = __dp4a(static_cast<int>(e[8 * w + 0]), static_cast<int>(a.x), acc[0]);
        acc[1] = __dp4a(static_cast<int>(e[8 * w + 1]), static_cast<int>(a.y), acc[1]);
        acc[2] = __dp4a(static_cast<int>(e[8 * w + 2]), static_cast<int>(a.z), acc[2]);
        acc[3] = __dp4a(static_cast<int>(e[8 * w + 3]), static_cast<int>(a.w), acc[3]);
        acc[0] = __dp4a(static_cast<int>(e[8 * w + 4]), static_cast<int>(b.x), acc[0]);
        acc[1] = __dp4a(static_cast<int>(e[8 * w + 5]), static_cast<int>(b.y), acc[1]);
        acc[2] = __dp4a(static_cast<int>(e[8 * w + 6]), static_cast<int>(b.z), acc[2]);
        acc[3] = __dp4a(static_cast<int>(e[8 * w + 7]), static_cast<int>(b.w), acc[3]);
    }
    return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// Unsigned-by-signed byte dot product: sum of a's 4 unsigned bytes times b's 4 signed bytes,
// plus c (PTX dp4a.u32.s32).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// The same sum for D > 128, where the whole split code would not fit in registers. Each
// 128-dim group of the code is used where it lies in the staged tile: the code word's bits s,
// s + 8, s + 16, s + 24 are masked in place (x & (0x01010101 << s), bytes 0 or 2^s), so
// dp4a over unsigned bytes gives 2^s times the plane's partial sum; accumulator s collects
// plane s and is shifted back once at the end (exact: |2^s * sum| <= 2^7 * 1024 * 128 <
// 2^31). One logic op and one dp4a per 4 dimensions, instead of a shift, a mask and a dp4a.
#ifndef CORA_SCAN_DP4A_WIDE
#define CORA_SCAN_DP4A_WIDE 1
#endif
constexpr bool kScanDp4aWide = CORA_SCAN_DP4A_WIDE != 0;
// cw: the vector's code words in the staged tile (group g at cw[g * stride]).
template <int G16>
__device__ __forceinline__ int ip_int_from_bytes_grouped(const uint4 *__restrict__ cw, int stride,
                                                         const uint32_t *__restrict__ Q) {
    int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll 1
    for (int g = 0; g < G16; ++g) {  // rolled: one group's query words in registers at a time
        const uint4 c = cw[g * stride];
        const uint32_t x[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int w = 4 * g + t;
            const uint4 a = *reinterpret_cast<const uint4 *>(Q + 8 * w);
            const uint4 b = *reinterpret_cast<const uint4 *>(Q + 8 * w + 4);
            const uint32_t qa[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int s = 0; s < 8; ++s)
                acc[s] = dp4a_us(x[t] & (0x01010101u << s), qa[s], acc[s]);
        }
    }
    return ((acc[0] + (acc[1] >> 1)) + ((acc[2] >> 2) + (acc[3] >> 3))) +
           (((acc[4] >> 4) + (acc[5] >> 5)) + ((acc[6] >> 6) + (acc[7] >> 7)));
}

// Copies a query's two's-complement bit-planes into shared memory as offset-binary planes
// (plane 7 inverted), the form ip_int_from_planes consumes.
__device__ __forceinline__ uint32_t offset_binary_word(uint32_t w, int word_index, int W4) {
    return word_index >= 7 * W4 ? ~w : w;
}

// ---- LUT estimator ---------------------------------------------------------------
// ip1 of one code from a pair's tables T (fp32, 16 per nibble group, shared memory): the
// reference's order of additions (vanguard_lut_inner_product, filter_kernels.cuh:283-306).
// Padding words (dims past D) meet zero entries: adding +0 to a sum that started at +0
// leaves it unchanged, so they need no test.
template <int G16>
__device__ __forceinline__ float ip_from_lut(const uint4 (&code)[G16], const float *__restrict__ T) {
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
    for (int g = 0; g < G16; ++g) {
        const uint32_t x[4] = {code[g].x, code[g].y, code[g].z, code[g].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float *Tw = T + (4 * g + t) * 128;  // word 4g + t: nibble groups 8w .. 8w + 7
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                acc0 = __fadd_rn(acc0, Tw[n * 16 + ((x[t] >> (28 - 4 * n)) & 0xFu)]);
                acc1 = __fadd_rn(acc1, Tw[(n + 1) * 16 + ((x[t] >> (24 - 4 * n)) & 0xFu)]);
            }
        }
    }
    return __fadd_rn(acc0, acc1);
}

// ip_from_lut for long codes (G16 >= 3): the code words are read from the staged tile group
// by group (cw: the vector's words, group g at cw[g * stride]) in a rolled loop, so the
// unrolled form's registers (and spills) are not needed; the same additions in the same order.
template <int G16>
__device__ __forceinline__ float ip_from_lut_grouped(const uint4 *__restrict__ cw, int stride,
                                                     const float *__restrict__ T) {
    float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 1
    for (int g = 0; g < G16; ++g) {
        const uint4 c = cw[g * stride];
        const uint32_t x[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float *Tw = T + (4 * g + t) * 128;
#pragma unroll
            for (int n = 0; n < 8; n += 2) {
                acc0 = __fadd_rn(acc0, Tw[n * 16 + ((x[t] >> (28 - 4 * n)) & 0xFu)]);
                acc1 = __fadd_rn(acc1, Tw[(n + 1) * 16 + ((x[t] >> (24 - 4 * n)) & 0xFu)]);
            }
        }
    }
    return __fadd_rn(acc0, acc1);
}
// G16 from which the LUT scans take ip_from_lut_grouped
constexpr int kLutGroupedFrom = 3;

// Widens query q's fp16 tables (4 D halves) into dst (kLutFloats fp32, zero past 4 D), one
// 16-byte load per thread and step; the calling threads cover [tid0, tid0 + nthreads).
template <int G16>
__device__ __forceinline__ void stage_lut(float *__restrict__ dst, const __half *__restrict__ lut,
                                          int q, int D, int tid0, int nthreads) {
    constexpr int LT = ScanShape<G16>::kLutFloats;
    const uint4 *src = reinterpret_cast<const uint4 *>(lut + (size_t)q * 4 * D);
    for (int i = tid0; i < LT / 8; i += nthreads) {
        float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
        if (8 * i < 4 * D) {
            const uint4 u = __ldg(src + i);
            const __half2 *h = reinterpret_cast<const __half2 *>(&u);
            const float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
            const float2 c = __half22float2(h[2]), d = __half22float2(h[3]);
            lo = make_float4(a.x, a.y, b.x, b.y);
            hi = make_float4(c.x, c.y, d.x, d.y);
        }
        reinterpret_cast<float4 *>(dst)[2 * i] = lo;
        reinterpret_cast<float4 *>(dst)[2 * i + 1] = hi;
    }
}

__device__ __forceinline__ float lower_bound_dist(float4 f, float ip1, float g, float k1,
                                                  float gerr) {
    const float a = __fadd_rn(f.x, g);
    const float b = __fmul_rn(f.y, __fadd_rn(ip1, k1));
    const float e = __fmul_rn(f.z, gerr);
    return __fsub_rn(__fadd_rn(a, b), e);
}

// Warp-aggregated append of a candidate record to query q's slice: one atomic per warp
// and query (the warp-ballot compaction of survivors).
__device__ __forceinline__ void emit_candidate(const SearchView &sv, bool cand, int q,
                                               uint64_t rec, int lane) {
    const uint32_t mask = __ballot_sync(0xffffffffu, cand);
    if (!mask) return;
    const int leader = __ffs(mask) - 1;
    uint32_t slot0 = 0;
    if (lane == leader) slot0 = atomicAdd(sv.cand_cnt + q, __popc(mask));
    slot0 = __shfl_sync(0xffffffffu, slot0, leader);
    if (cand) {
        const uint32_t slot = slot0 + __popc(mask & ((1u << lane) - 1u));
        if (slot < static_cast<uint32_t>(sv.cap))
            sv.cand_rec[(size_t)q * sv.cap + slot] = rec;
        else
            atomicOr(sv.err, kDevCandidateOverflow);
    }
}

// Writes the seeds of one vanguard pair (keys sorted ascending in s_keys[0, nkeep)) and its
// boundary key (kKeyMax when every candidate became a seed). Thread 0 reserves the slots.
__device__ __forceinline__ void write_seeds(const SearchView &sv, int q, int r, int total,
                                            const uint64_t *s_keys, uint32_t *s_base) {
    const int nkeep = min(total, sv.keep);
    if (threadIdx.x == 0) {
        *s_base = nkeep ? atomicAdd(sv.cand_cnt + q, static_cast<uint32_t>(nkeep)) : 0u;
        sv.bound[(size_t)q * sv.veff + r] = total <= sv.keep ? kKeyMax : s_keys[sv.keep - 1];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nkeep; i += blockDim.x) {
        const uint32_t slot = *s_base + i;
        const uint32_t gid = static_cast<uint32_t>(s_keys[i] & 0xFFFFFFFFu);
        if (slot < static_cast<uint32_t>(sv.cap))
            sv.cand_rec[(size_t)q * sv.cap + slot] = gid | (static_cast<uint64_t>(r) << 32);
        else
            atomicOr(sv.err, kDevCandidateOverflow);
    }
}

// ---- grouped scan: persistent CTAs over (cluster, <= 32 pairs) items -----------------
// kWriteLows: store every low in the pair's slice of sv.lows (vanguard pass).
// otherwise:  emit candidates low < T1 (main pass; vanguard seeds are skipped through the
//             boundary key when vanguard pairs are rescanned). A pair is dropped from an
//             item, and from each 32-vector chunk (one warp of a tile), whose factor range
//             proves every low >= T1 (range_at_least): no tile is loaded for an item that
//             keeps no pair, and a warp evaluates only the pairs its chunk keeps.
// kLut: ip1 from the LUT estimator (each pair's tables staged in shared memory as fp32;
// items hold at most ScanShape::kLutPairs pairs).
template <int G16, bool kWriteLows, bool kLut>
__global__ void __launch_bounds__(kScanThreads, CORA_SCAN_MINB(G16)) scan_kernel(
    IndexView ix, SearchView sv, const ScanItem *__restrict__ items,
    const uint32_t *__restrict__ n_items_ptr, const uint32_t *__restrict__ pairs,
    int *__restrict__ item_counter) {
    using Sh = ScanShape<G16>;
    constexpr int TV = Sh::kScanTV, W4 = Sh::W4, S = Sh::kStages, SE = Sh::kScanStageEntries;
    // query words: byte words for dp4a (the split code is 32 * G16 registers, so only for
    // D <= 128), offset-binary bit-planes otherwise; both are 8 * W4 words per query. With
    // the LUT estimator: kLutFloats fp32 table entries per pair.
    constexpr bool kBytes = kScanDp4a && G16 == 1 && !kLut;
    // D > 128: byte words too, the code split group by group (ip_int_from_bytes_grouped)
    constexpr bool kBytesWide = kScanDp4a && kScanDp4aWide && G16 > 1 && !kLut;
    constexpr int kQB = kLut ? Sh::kLutFloats : 8 * W4;  // 32-bit words per pair
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4 *stage = reinterpret_cast<uint4 *>(smem_raw);
    uint32_t *s_planes = reinterpret_cast<uint32_t *>(stage + S * SE);
    __shared__ __align__(8) uint64_t bars[S];
    __shared__ uint64_t s_bnd[kMaxPairsPerItem];  // main pass: each pair's seed boundary key
    __shared__ float *s_lp[kMaxPairsPerItem];     // lows pass: each pair's lows slice
    // per pair: {width, g, k1, sqrt(max(g, 0))} (one 16-byte read per evaluation)
    __shared__ float4 s_par[kMaxPairsPerItem];
    __shared__ float s_T1[kMaxPairsPerItem], s_M[kMaxPairsPerItem];
    __shared__ int s_q[kMaxPairsPerItem], s_r[kMaxPairsPerItem];
    __shared__ int s_item, s_abort;
    __shared__ uint32_t s_keep;  // main pass: the item's pairs that some vector may need
    __shared__ unsigned long long s_lbase;  // lows pass: this item's slices (~0ull: no room)

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) mbar_init(&bars[i], 1);
        fence_barrier_init();
        s_abort = 0;
    }
    __syncthreads();
    const uint32_t n_items = *n_items_ptr;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t phase = 0;  // bit i: parity of the next phase of bars[i]
    while (true) {
        if (threadIdx.x == 0) s_item = atomicAdd(item_counter, 1);
        __syncthreads();
        const int it = s_item;
        if (it >= static_cast<int>(n_items)) break;
        const ScanItem item = items[it];
        const int c = static_cast<int>(item.cluster);
        const uint32_t s = ix.cl_start[c];
        const int n = static_cast<int>(ix.cl_size[c]);
        const int pc = static_cast<int>(item.pair_count);
        const size_t cbase = (size_t)(G16 + 1) * s;
        const int ntiles = (n + TV - 1) / TV;
        const uint32_t chunk0 = kWriteLows ? 0u : ix.cl_chunk[c];
        if (kWriteLows) {
            if (threadIdx.x == 0) {
                const unsigned long long need =
                    (unsigned long long)pc * lows_slice(static_cast<uint32_t>(n));
                unsigned long long b = atomicAdd(sv.lows_top, need);
                if (b + need > sv.lows_cap) {
                    atomicOr(sv.err, kDevCandidateOverflow);
                    b = ~0ull;
                }
                s_lbase = b;
            }
            __syncthreads();
        }
        if (threadIdx.x < pc) {
            const uint32_t pr = pairs[item.pair_begin + threadIdx.x];
            const int q = static_cast<int>(pr >> 16), r = static_cast<int>(pr & 0xFFFFu);
            const float g = sv.probe_g[(size_t)q * sv.nprobe + r];
            const float ga = sv.probe_ga[(size_t)q * sv.nprobe + r];
            const QueryScalars qs = sv.scal[q];
            s_q[threadIdx.x] = q;
            s_r[threadIdx.x] = r;
            s_par[threadIdx.x] = make_float4(qs.width, ga, qs.k1, __fsqrt_rn(fmaxf(g, 0.0f)));
            if (kWriteLows) {
                // slice of this vanguard pair (offset 0 when the buffer is full: the search
                // reports the overflow, and the readers of the slice stay in bounds)
                const unsigned long long b = s_lbase;
                const uint64_t off =
                    b == ~0ull ? 0ull
                               : b + (uint64_t)threadIdx.x * lows_slice(static_cast<uint32_t>(n));
                sv.vg_off[(size_t)q * sv.veff + r] = off;
                s_lp[threadIdx.x] = sv.lows + off;
                if (b != ~0ull)  // the slice's padding reads as +inf (never below a threshold)
                    for (uint32_t p = n; p < lows_slice(static_cast<uint32_t>(n)); ++p)
                        sv.lows[off + p] = __int_as_float(0x7f800000);
            } else {
                s_T1[threadIdx.x] = sv.T1[q];
                s_M[threadIdx.x] = sv.ipm[q];
                s_bnd[threadIdx.x] = r < sv.veff ? sv.bound[(size_t)q * sv.veff + r] : 0ull;
            }
        }
        __syncthreads();
        uint32_t keep = pc == 32 ? ~0u : (1u << pc) - 1u;
        if (kWriteLows) {
            if (s_lbase == ~0ull) continue;  // no room for the lows: the search fails anyway
            if (threadIdx.x == 0)  // the first S - 1 tiles go out at once
                for (int u = 0; u < S - 1 && u < ntiles; ++u)
                    issue_tile<G16, TV>(stage + u * SE, &bars[u], ix.scan4, cbase, n, u * TV,
                                        min(TV, n - u * TV));
        } else {
            if (warp == 0) {
                bool need = false;
                if (lane < pc) {
                    const float4 pj = s_par[lane];
                    need = !range_at_least(ix.cl_range[c], pj.y, s_M[lane], pj.w, s_T1[lane]);
                }
                const uint32_t m = __ballot_sync(0xffffffffu, need);
                if (lane == 0) s_keep = m;
            }
            __syncthreads();
            keep = s_keep;
            if (keep == 0) continue;  // no vector of the cluster can be a candidate
            if (threadIdx.x == 0)
                for (int u = 0; u < S - 1 && u < ntiles; ++u)
                    issue_tile<G16, TV>(stage + u * SE, &bars[u], ix.scan4, cbase, n, u * TV,
                                        min(TV, n - u * TV));
        }
        if constexpr (kLut) {
            // one warp per pair in turn
            for (int j = warp; j < pc; j += kScanThreads / 32)
                stage_lut<G16>(reinterpret_cast<float *>(s_planes) + j * kQB, sv.lut, s_q[j],
                               ix.D, lane, 32);
        } else {
            for (int i = threadIdx.x; i < pc * kQB; i += blockDim.x) {
                const int j = i / kQB, r = i - j * kQB;
                const uint32_t *pl = sv.planes + (size_t)s_q[j] * 8 * W4;
                s_planes[i] = (kBytes || kBytesWide) ? query_byte_word(pl, r >> 3, r & 7, W4)
                                                     : offset_binary_word(pl[r], r, W4);
            }
        }
        __syncthreads();
        for (int t = 0; t < ntiles; ++t) {
            const int b = t % S;
            const int v0 = t * TV, tv = min(TV, n - v0);
            if (!mbar_wait_bounded(&bars[b], (phase >> b) & 1u, sv.err)) s_abort = 1;
            phase ^= 1u << b;
            __syncthreads();
            if (s_abort) {
                // let the copies still in flight (tiles t .. t + S - 2) land before exiting
                if (threadIdx.x == 0)
                    for (int u = t; u < t + S - 1 && u < ntiles; ++u)
                        mbar_wait_bounded(&bars[u % S], ((phase >> (u % S)) & 1u) ^ (u == t),
                                          sv.err);
                return;
            }
            if (threadIdx.x == 0 && t + S - 1 < ntiles) {  // into the slot tile t - 1 freed
                const int u = t + S - 1;
                issue_tile<G16, TV>(stage + (u % S) * SE, &bars[u % S], ix.scan4, cbase, n,
                                    u * TV, min(TV, n - u * TV));
            }
            const uint4 *sb = stage + b * SE;
            constexpr int V = Sh::VPT;
            // the pairs this warp's chunks (vectors v0 + 256 v + 32 warp ..) keep
            uint32_t wkeep = keep;
            if (!kWriteLows) {
                static_assert(TV == kScanThreads * V, "thread t evaluates vectors t + 256 v");
                wkeep = 0;
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const int k = (v0 + v * kScanThreads) / 32 + warp;
                    bool need = false;
                    if (k * 32 < n && lane < pc && ((keep >> lane) & 1u)) {
                        const float4 pj = s_par[lane];
                        need = !range_at_least(__ldg(ix.chunk_range + chunk0 + k), pj.y,
                                               s_M[lane], pj.w, s_T1[lane]);
                    }
                    wkeep |= __ballot_sync(0xffffffffu, need);
                }
            }
            // every thread evaluates V vectors of the tile against each query in turn, so a
            // query's words are read from shared memory once per V vectors
            for (int vb = 0; vb < tv; vb += V * kScanThreads) {
                uint4 code[V][G16];
                float4 f[V];
                int bias[V];
                uint32_t e[V][kBytes ? 32 * G16 : 1];
                (void)bias;
                bool valid[V];
#pragma unroll
                for (int v = 0; v < V; ++v) {
                    const int i = vb + v * kScanThreads + threadIdx.x;
                    valid[v] = i < tv;
                    f[v] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int gg = 0; gg < G16; ++gg)
                        code[v][gg] = valid[v] ? sb[gg * TV + i] : make_uint4(0, 0, 0, 0);
                    if (valid[v]) {
                        const uint4 fr = sb[G16 * TV + i];
                        f[v] = make_float4(__uint_as_float(fr.x), __uint_as_float(fr.y),
                                           __uint_as_float(fr.z), 0.0f);
                    }
                    if constexpr (kBytes)
                        split_code_bytes<G16>(code[v], e[v]);
                    else if constexpr (!kLut && !kBytesWide)
                        bias[v] = code_bias<G16>(code[v]);
                }
                // lows pass: every pair in order; main pass: the pairs this warp's chunk keeps
                for (uint32_t mj = wkeep, jj = 0; kWriteLows ? jj < static_cast<uint32_t>(pc) : mj != 0;
                     mj &= mj - 1u, ++jj) {
                    const int j = kWriteLows ? static_cast<int>(jj) : __ffs(mj) - 1;
                    const uint32_t *P = s_planes + j * kQB;
#pragma unroll
                    for (int v = 0; v < V; ++v) {
                        const int i = vb + v * kScanThreads + threadIdx.x;
                        const float4 pj = s_par[j];
                        float ip1;
                        if constexpr (kLut) {
                            if constexpr (G16 >= kLutGroupedFrom)  // (V == 1)
                                ip1 = ip_from_lut_grouped<G16>(sb + i, TV,
                                                               reinterpret_cast<const float *>(P));
                            else
                                ip1 = ip_from_lut<G16>(code[v], reinterpret_cast<const float *>(P));
                        } else {
                            int ip;
                            if constexpr (kBytes)
                                ip = ip_int_from_bytes<G16>(e[v], P);
                            else if constexpr (kBytesWide)  // (V == 1 for G16 > 1)
                                ip = ip_int_from_bytes_grouped<G16>(sb + i, TV, P);
                            else
                                ip = ip_int_from_planes<G16>(code[v], P, bias[v]);
                            // ip1 = width * ip_int (+ 0 in the reference: width >= 1e-30 and
                            // |ip_int| >= 1 or ip_int = 0 give a normal or +0 product, which
                            // the addition of 0 leaves unchanged)
                            ip1 = __fmul_rn(pj.x, (float)ip);
                        }
                        const float low = lower_bound_dist(f[v], ip1, pj.y, pj.z, pj.w);
                        if (kWriteLows) {
                            if (valid[v]) s_lp[j][v0 + i] = low;
                        } else {
                            const uint32_t gid = s + static_cast<uint32_t>(v0 + i);
                            const bool cand =
                                valid[v] && (low < s_T1[j]) && (make_key(low, gid) > s_bnd[j]);
                            emit_candidate(sv, cand, s_q[j],
                                           gid | (static_cast<uint64_t>(s_r[j]) << 32), lane);
                        }
                    }
                }
            }
            __syncthreads();  // stage buffer b is free again
        }
    }
}

// ---- lows mode: per vanguard pair seed selection and candidate filtering -------------
// One CTA per vanguard pair: seeds are the best `keep` keys among low < T0. The pair's lows
// are staged in shared memory when they fit (kSelectStage floats), so the radix passes
// read them from there. Dynamic shared memory: next_pow2(keep) keys + kSelectStage floats.
// With `list` the CTAs serve the pairs queued there (list[0] pairs at list[1..]) in a
// grid-stride loop; without it CTA i serves vanguard pair i.
constexpr uint32_t kSelectStage = 8192;
__device__ void select_pair_block(const IndexView &ix, const SearchView &sv,
                                  const uint8_t *owned, int pi, uint64_t *s_keys, int *scratch,
                                  int *s_total, uint32_t *s_base);
__global__ void __launch_bounds__(256) vanguard_select_kernel(IndexView ix, SearchView sv,
                                                              const uint8_t *__restrict__ owned,
                                                              const uint32_t *__restrict__ list) {
    extern __shared__ uint64_t s_keys[];
    __shared__ int scratch[256 + 3];
    __shared__ int s_total;
    __shared__ uint32_t s_base;
    if (!list) {
        select_pair_block(ix, sv, owned, blockIdx.x, s_keys, scratch, &s_total, &s_base);
        return;
    }
    const uint32_t count = list[0];
    for (uint32_t j = blockIdx.x; j < count; j += gridDim.x) {
        select_pair_block(ix, sv, owned, static_cast<int>(list[1 + j]), s_keys, scratch, &s_total,
                          &s_base);
        __syncthreads();
    }
}

__device__ void select_pair_block(const IndexView &ix, const SearchView &sv,
                                  const uint8_t *owned, int pi, uint64_t *s_keys, int *scratch,
                                  int *s_total_p, uint32_t *s_base_p) {
    int &s_total = *s_total_p;
    const int q = pi / sv.veff, r = pi % sv.veff;
    const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
    if (owned && !owned[c]) return;
    const uint32_t s = ix.cl_start[c];
    const uint32_t n = ix.cl_size[c];
    const float *Lg = sv.lows + sv.vg_off[pi];
    float *s_lows = reinterpret_cast<float *>(s_keys + next_pow2(sv.keep));
    const bool staged = n <= kSelectStage;
    const float *L = staged ? s_lows : Lg;
    const float T0 = sv.T0[q];
    if (threadIdx.x == 0) s_total = 0;
    __syncthreads();
    int mine = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float l = Lg[i];
        if (staged) s_lows[i] = l;
        mine += l < T0;
    }
    atomicAdd(&s_total, mine);
    __syncthreads();
    auto key_at = [&](uint32_t i) -> uint64_t {
        const float l = L[i];
        return l < T0 ? make_key(l, s + i) : kKeyMax;
    };
    block_select_smallest(key_at, n, sv.keep, s_keys, scratch);
    write_seeds(sv, q, r, s_total, s_keys, s_base_p);
}

constexpr int kLowsUnroll = 4;  // float4 lows loaded per lane before they are processed

// Loads lows 4 * (i4 .. i4 + 32 * (kLowsUnroll - 1)) of a slice as float4 (slices are
// 16-byte aligned and padded with +inf to a multiple of 4); float4s past the slice read as
// +inf.
__device__ __forceinline__ void load_lows4(const float4 *__restrict__ L4, uint32_t n,
                                           uint32_t i4, float (&l)[4 * kLowsUnroll]) {
    const float inf = __int_as_float(0x7f800000);
#pragma unroll
    for (int t = 0; t < kLowsUnroll; ++t) {  // all loads first: one round trip per batch
        const uint32_t j4 = i4 + 32 * t;
        float4 v = make_float4(inf, inf, inf, inf);
        if (4 * j4 < n) v = __ldg(L4 + j4);
        l[4 * t + 0] = v.x;
        l[4 * t + 1] = v.y;
        l[4 * t + 2] = v.z;
        l[4 * t + 3] = v.w;
    }
}
// Slice index of bit e of a lane's batch mask (element e of load_lows4's array).
__device__ __forceinline__ uint32_t lows_index(uint32_t b4, int lane, int e) {
    return 4 * (b4 + lane + 32 * (e >> 2)) + (e & 3);
}

// The vanguard pairs the lows filter must read: owned by this shard and not proven
// candidate-free against T1 by their cluster's factor range (range_at_least). Appended to
// list[1..] (count in list[0], zeroed by the caller) with one atomic per warp.
__global__ void __launch_bounds__(256) filter_list_kernel(IndexView ix, SearchView sv,
                                                          const uint8_t *__restrict__ owned,
                                                          uint32_t *__restrict__ list) {
    const int pi = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    bool keep = false;
    if (pi < sv.nq * sv.veff) {
        const int q = pi / sv.veff, r = pi % sv.veff;
        const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
        if (!owned || owned[c]) {
            const float g = sv.probe_g[(size_t)q * sv.nprobe + r];
            const float ga = sv.probe_ga[(size_t)q * sv.nprobe + r];
            keep = !range_at_least(ix.cl_range[c], ga, sv.ipm[q], __fsqrt_rn(fmaxf(g, 0.0f)),
                                   sv.T1[q]);
        }
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, keep);
    if (!mask) return;
    uint32_t base = 0;
    if (lane == 0) base = atomicAdd(list, __popc(mask));
    base = __shfl_sync(0xffffffffu, base, 0);
    if (keep) list[1 + base + __popc(mask & ((1u << lane) - 1u))] = static_cast<uint32_t>(pi);
}

// One warp per listed vanguard pair (filter_list_kernel; 8 per CTA, warps past the list's
// count exit): candidates low < T1 that are not seeds (key > boundary), read from the
// pair's stored lows.
__global__ void __launch_bounds__(256) vanguard_filter_kernel(IndexView ix, SearchView sv,
                                                              const uint32_t *__restrict__ list) {
    const int lane = threadIdx.x & 31;
    const uint32_t li = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (li >= list[0]) return;  // warp-uniform
    const int pi = static_cast<int>(list[1 + li]);
    const int q = pi / sv.veff, r = pi % sv.veff;
    const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
    const uint32_t s = ix.cl_start[c];
    const uint32_t n = ix.cl_size[c];
    const float T1 = sv.T1[q];
    const float4 *L4 = reinterpret_cast<const float4 *>(sv.lows + sv.vg_off[pi]);
    const uint64_t bnd = sv.bound[(size_t)q * sv.veff + r];
    const uint64_t rtag = static_cast<uint64_t>(r) << 32;
    for (uint32_t b4 = 0; 4 * b4 < n; b4 += 32 * kLowsUnroll) {
        float l[4 * kLowsUnroll];
        load_lows4(L4, n, b4 + lane, l);
        // bit e: element e of this lane's batch is below T1 and not a seed (key above the
        // boundary; the padding reads as +inf)
        uint32_t take = 0;
#pragma unroll
        for (int e = 0; e < 4 * kLowsUnroll; ++e)
            if (l[e] < T1 && make_key(l[e], s + lows_index(b4, lane, e)) > bnd) take |= 1u << e;
        // one warp prefix sum and one slot reservation per batch
        const uint32_t mine = __popc(take);
        const uint32_t incl = warp_inclusive_sum(mine, lane);
        const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
        if (total == 0) continue;
        uint32_t base = 0;
        if (lane == 31) base = atomicAdd(sv.cand_cnt + q, total);
        uint32_t slot = __shfl_sync(0xffffffffu, base, 31) + incl - mine;
        for (uint32_t m = take; m; m &= m - 1, ++slot) {
            const uint32_t i = lows_index(b4, lane, __ffs(m) - 1);
            if (slot < static_cast<uint32_t>(sv.cap))
                sv.cand_rec[(size_t)q * sv.cap + slot] = (s + i) | rtag;
            else
                atomicOr(sv.err, kDevCandidateOverflow);
        }
    }
}

// ---- warp-level seed selection for keep <= 32 -----------------------------------------
constexpr int kWarpSelectMax = 128;  // largest `keep` handled one warp per pair
constexpr int kWarpSelectBuf = 256;  // keys at or below the first threshold a warp may hold

// One warp per vanguard pair (8 per CTA), keep <= 32 T (T <= 4). Each lane keeps its T
// smallest lows; the keep-th smallest of those 32 T values bounds the keep-th smallest key
// from above (keep of them lie at or below it), so every seed is among the keys at or below
// it; those (normally little more than keep) are collected and sorted. A pair whose
// collection exceeds kWarpSelectBuf is queued in fallback[1..] (count in fallback[0]) for
// vanguard_select_kernel.
template <int T>
__global__ void __launch_bounds__(256) vanguard_select_warp_kernel(
    IndexView ix, SearchView sv, const uint8_t *__restrict__ owned,
    uint32_t *__restrict__ fallback) {
    __shared__ uint64_t buf[8][kWarpSelectBuf];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int pi = blockIdx.x * 8 + w;
    if (pi >= sv.nq * sv.veff) return;  // warp-uniform
    const int q = pi / sv.veff, r = pi % sv.veff;
    const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
    if (owned && !owned[c]) return;
    const uint32_t s = ix.cl_start[c];
    const uint32_t n = ix.cl_size[c];
    const float4 *L4 = reinterpret_cast<const float4 *>(sv.lows + sv.vg_off[pi]);
    const float T0 = sv.T0[q];
    const int S = sv.keep;
    // Pass 1: each lane's T smallest lows (branch-free insertion; NaN lows drop out of
    // fminf / fmaxf). tau_f, the S-th smallest of the 32 T values, bounds the seeds: when
    // tau_f < T0, S values at or below it are lows below T0, so the S smallest keys all have
    // low <= tau_f; when tau_f >= T0 every low < T0 is collected.
    const float inf = __int_as_float(0x7f800000);
    float mn[T];
#pragma unroll
    for (int t = 0; t < T; ++t) mn[t] = inf;
    for (uint32_t b4 = 0; 4 * b4 < n; b4 += 32 * kLowsUnroll) {
        float l[4 * kLowsUnroll];
        load_lows4(L4, n, b4 + lane, l);
#pragma unroll
        for (int e = 0; e < 4 * kLowsUnroll; ++e) {
            float x = fminf(l[e], inf);  // NaN -> inf: an inserted NaN would duplicate a value
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const float lo = fminf(mn[t], x);
                x = fmaxf(mn[t], x);
                mn[t] = lo;
            }
        }
    }
    uint64_t *b = buf[w];
    float tau_f;
    if (T == 1) {
        tau_f = unord_f32(static_cast<uint32_t>(
            __shfl_sync(0xffffffffu, warp_sort_lane_keys(make_key(mn[0], lane), lane), S - 1) >> 32));
    } else {
#pragma unroll
        for (int t = 0; t < T; ++t) b[lane * T + t] = make_key(mn[t], lane * T + t);
        __syncwarp();
        warp_sort_smem(b, 32 * T, lane);
        tau_f = unord_f32(static_cast<uint32_t>(b[S - 1] >> 32));
        __syncwarp();
    }
    // Pass 2: count the lows < T0 and collect every key with low < T0 and low <= tau_f (-0
    // and +0 compare equal here, so the set contains every key the exact bound would take)
    const float *L = sv.lows + sv.vg_off[pi];
    uint32_t m = 0, cnt = 0;
    for (uint32_t b4 = 0; 4 * b4 < n; b4 += 32 * kLowsUnroll) {
        float l[4 * kLowsUnroll];
        load_lows4(L4, n, b4 + lane, l);
        uint32_t take = 0;
#pragma unroll
        for (int e = 0; e < 4 * kLowsUnroll; ++e) {
            const bool below = l[e] < T0;
            cnt += below ? 1u : 0u;
            take |= (below && l[e] <= tau_f ? 1u : 0u) << e;
        }
        const uint32_t mine = __popc(take);
        const uint32_t incl = warp_inclusive_sum(mine, lane);
        const uint32_t got = __shfl_sync(0xffffffffu, incl, 31);
        uint32_t pos = m + incl - mine;
        for (uint32_t mm = take; mm; mm &= mm - 1, ++pos) {
            const uint32_t i = lows_index(b4, lane, __ffs(mm) - 1);
            if (pos < static_cast<uint32_t>(kWarpSelectBuf)) b[pos] = make_key(L[i], s + i);
        }
        m += got;
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, cnt);
    if (m > static_cast<uint32_t>(sv.warp_select_limit)) {
        if (lane == 0) fallback[1 + atomicAdd(fallback, 1u)] = static_cast<uint32_t>(pi);
        return;
    }
    int sort_n = 32;
    while (sort_n < static_cast<int>(m)) sort_n <<= 1;
    for (int i = m + lane; i < sort_n; i += 32) b[i] = kKeyMax;
    __syncwarp();
    warp_sort_smem(b, sort_n, lane);
    // the collection holds every seed (at least min(total, S) keys); a shortfall would mean
    // a broken bound, reported instead of emitting ids that are not in the index
    int nkeep = min(static_cast<int>(total), S);
    if (static_cast<int>(m) < nkeep) {
        if (lane == 0) atomicOr(sv.err, kDevBadInput);
        nkeep = static_cast<int>(m);
    }
    uint32_t slot0 = 0;
    if (lane == 0) {
        slot0 = nkeep ? atomicAdd(sv.cand_cnt + q, static_cast<uint32_t>(nkeep)) : 0u;
        sv.bound[(size_t)q * sv.veff + r] = total <= static_cast<uint32_t>(S) ? kKeyMax : b[S - 1];
    }
    slot0 = __shfl_sync(0xffffffffu, slot0, 0);
    for (int i = lane; i < nkeep; i += 32) {
        const uint32_t slot = slot0 + i;
        const uint32_t gid = static_cast<uint32_t>(b[i] & 0xFFFFFFFFu);
        if (slot < static_cast<uint32_t>(sv.cap))
            sv.cand_rec[(size_t)q * sv.cap + slot] = gid | (static_cast<uint64_t>(r) << 32);
        else
            atomicOr(sv.err, kDevCandidateOverflow);
    }
}

// ---- rescan mode: one CTA per vanguard pair scans the cluster and keeps its seeds ----
template <int G16, bool kLut>
__global__ void __launch_bounds__(kScanThreads) vanguard_rescan_kernel(
    IndexView ix, SearchView sv, int sort_n, const uint8_t *__restrict__ owned) {
    using Sh = ScanShape<G16>;
    constexpr int TV = Sh::TV, W4 = Sh::W4;
    constexpr int kQB = kLut ? Sh::kLutFloats : 8 * W4;  // query words (see scan_kernel)
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4 *stage = reinterpret_cast<uint4 *>(smem_raw);                      // [2][(G16+1)TV]
    uint32_t *s_planes = reinterpret_cast<uint32_t *>(stage + 2 * Sh::kStageEntries);
    uint64_t *s_keys = reinterpret_cast<uint64_t *>(s_planes + kQB);        // sort_n
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ int n_staged, n_total, s_abort;
    __shared__ uint64_t thresh;
    __shared__ uint32_t s_base;

    const int pi = blockIdx.x;
    const int q = pi / sv.veff, r = pi % sv.veff;
    const int c = sv.probe_ids[(size_t)q * sv.nprobe + r];
    if (owned && !owned[c]) return;
    const float g = sv.probe_g[(size_t)q * sv.nprobe + r];
    const float ga = sv.probe_ga[(size_t)q * sv.nprobe + r];
    const uint32_t s = ix.cl_start[c];
    const int n = static_cast<int>(ix.cl_size[c]);
    const QueryScalars qs = sv.scal[q];
    const float T0 = sv.T0[q];
    const float gerr = __fsqrt_rn(fmaxf(g, 0.0f));
    const size_t cbase = (size_t)(G16 + 1) * s;

    if constexpr (kLut) {
        stage_lut<G16>(reinterpret_cast<float *>(s_planes), sv.lut, q, ix.D, threadIdx.x,
                       blockDim.x);
    } else {
        for (int i = threadIdx.x; i < 8 * W4; i += blockDim.x)
            s_planes[i] = offset_binary_word(sv.planes[(size_t)q * 8 * W4 + i], i, W4);
    }
    if (threadIdx.x == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
        n_total = 0;
        s_abort = 0;
    }
    BlockTopK tk{s_keys, sv.keep, TV, sort_n, &n_staged, &thresh};
    tk.init(kKeyMax);  // also synchronises the barrier init and the planes
    const int ntiles = (n + TV - 1) / TV;
    uint32_t phase[2] = {0, 0};
    if (threadIdx.x == 0 && ntiles > 0) issue_tile<G16>(stage, &bars[0], ix.scan4, cbase, n, 0, min(TV, n));
    for (int t = 0; t < ntiles; ++t) {
        const int b = t & 1;
        const int v0 = t * TV, tv = min(TV, n - v0);
        if (!mbar_wait_bounded(&bars[b], phase[b], sv.err)) s_abort = 1;
        phase[b] ^= 1;
        __syncthreads();
        if (s_abort) return;
        if (threadIdx.x == 0 && t + 1 < ntiles)
            issue_tile<G16>(stage + (b ^ 1) * Sh::kStageEntries, &bars[b ^ 1], ix.scan4, cbase, n,
                            v0 + TV, min(TV, n - v0 - TV));
        const uint4 *sb = stage + b * Sh::kStageEntries;
        for (int i = threadIdx.x; i < tv; i += blockDim.x) {
            uint4 code[G16];
#pragma unroll
            for (int gg = 0; gg < G16; ++gg) code[gg] = sb[gg * TV + i];
            const uint4 fr = sb[G16 * TV + i];
            const float4 f = make_float4(__uint_as_float(fr.x), __uint_as_float(fr.y),
                                         __uint_as_float(fr.z), 0.0f);
            float ip1;
            if constexpr (kLut && G16 >= kLutGroupedFrom) {
                ip1 = ip_from_lut_grouped<G16>(sb + i, TV, reinterpret_cast<const float *>(s_planes));
            } else if constexpr (kLut) {
                ip1 = ip_from_lut<G16>(code, reinterpret_cast<const float *>(s_planes));
            } else {
                const int ip = ip_int_from_planes<G16>(code, s_planes, code_bias<G16>(code));
                ip1 = __fadd_rn(__fmul_rn(qs.width, (float)ip), 0.0f);
            }
            const float low = lower_bound_dist(f, ip1, ga, qs.k1, gerr);
            if (low < T0) {
                atomicAdd(&n_total, 1);
                tk.offer(make_key(low, s + v0 + i));
            }
        }
        tk.flush(kKeyMax);  // includes the barrier that frees stage buffer b
    }
    write_seeds(sv, q, r, n_total, s_keys, &s_base);
}

}  // namespace cora
