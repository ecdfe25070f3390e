/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the IVF-RaBitQ search hot path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load this
 * library, and only as the checker. The product (libcoraanns_b200.so) never links it.
 *
 * It restates, single-threaded per query and in a fixed evaluation order, the arithmetic
 * of the reference's hybrid search path (paths within the reference project):
 *   rotation           src/search/hybrid.cu:436-440 (q' = q * P)
 *   query factors      src/search/query_kernels.cuh:73-94      (sumq, k1, kb)
 *   query bit-planes   src/search/query_kernels.cuh:117-189    (8-bit symmetric, Bq = 8)
 *   coarse distances   src/search/hybrid.cu:465-477 + select_k :485-493
 *   1-bit estimator    src/search/filter_kernels.cuh:79-114    (popcount ip_int)
 *   lower bound        src/search/filter_kernels.cuh:693-696 / index/estimator.hpp:65-70
 *   ex refinement      src/search/cpu_refinement.cpp:183-191   (8-bit code IP)
 *   7-bit decode       third_party/rabitq/.../utils/space.hpp:677-762, layout
 *                      third_party/rabitq/.../quantization/pack_excode.hpp:216-264
 *   top-k              src/search/cpu_refinement.cpp:202-230,269-283
 *   vanguard seeding   src/search/filter_kernels.cuh:308-468,470-582 (keep max(topk,20))
 *
 * Determinism contract (the CUDA kernels follow it operation for operation):
 *  - rotation and centroid distances accumulate in fp64 in ascending index order (fp64
 *    fma; products of two fp32 values are exact in fp64) and round once to fp32; sumq
 *    accumulates in fp64 over 32 strided lanes combined by an xor butterfly;
 *  - ip_int is exact integer arithmetic; ip1 = width * (float)ip_int; or, with the LUT
 *    estimator (lut_estimator = 1; query_kernels.cuh:199-221, filter_kernels.cuh:283-306),
 *    ip1 = acc0 + acc1 over fp16 table entries: entry (g, p) = half_rne(fp32 sum from 0 of
 *    the q' of dims 4g + i with bit 3 - i of p set, i ascending), and nibble n of code word
 *    w (bits 31 - 4n .. 28 - 4n) adds entry (8w + n, nibble) to acc0 (n even) or acc1 (n
 *    odd), in ascending (w, n) order, in fp32;
 *  - low / ex follow the reference's expression trees in fp32, round-to-nearest, with no
 *    contraction (built with -ffp-contract=off);
 *  - refinement follows the reference's expression (cpu_refinement.cpp:183-191,
 *    estimator.hpp:86-103): ex = (f_add_ex + g) + f_rescale_ex * ((2^ex_bits * ip1 + ip2)
 *    + kb), with ip1 = width * ip_int the scan's integer estimate of <q', b> (the exact_ip
 *    the reference's producers publish, filter_kernels.cuh:106) and ip2 = <q', u> over the
 *    decoded ex code u, one fp64 accumulation in ascending dimension order (exact
 *    products) rounded once (the reference sums in fp32 with AVX FMAs: ip2 agrees within
 *    1e-4 relative, tests/test_oracle.py);
 *  - opt-in (refine_full_code = 1): the full 8-bit code inner product ipT = <q', 128 b + u>
 *    in place of 128 * ip1 + ip2, one fp64 accumulation rounded once; it removes ip1's
 *    query-quantisation error, which the reference form multiplies by 128;
 *  - coarse probes are ordered by (g_add, cluster id); results by (ex, original id);
 *  - thresholds are static per phase (seeded T0, then T1 from the vanguard seeds), so the
 *    candidate set {v : low(v) < T} is a pure function of the inputs. The first
 *    max(vanguard, 1) probes keep their best max(k, 20) vectors by (low, gid) among
 *    low < T0 as seeds; T1 = min(T0, k-th smallest seed distance). The main phase scans
 *    every probe, skipping seeds, with candidates low < T1; results are the best k by
 *    (ex, id) among seeds and candidates with ex < T0.
 *
 * Inputs use the reference adapter's packed layout (src/index/search_data.cpp:45-123):
 * word-major 1-bit codes per cluster with bit (31-b) of word w holding dim 32w+b, float[N][3]
 * short factors, compact ex codes N x (D*ex_bits/8) and float[N][2] ex factors.
 */
#ifndef CORA_ORACLE_H
#define CORA_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t num, dim, padded_dim, nlist, ex_bits;
    const float *centroids;        /* nlist x D, rotated */
    const float *rotator;          /* dim x D, row-major */
    const uint32_t *short_data;    /* N x D/32, word-major per cluster */
    const float *short_factors;    /* N x 3: f_add, f_rescale, f_error */
    const uint8_t *long_codes;     /* N x D*ex_bits/8 */
    const float *ex_factors;       /* N x 2: f_add_ex, f_rescale_ex */
    const uint32_t *ids;           /* N original ids, cluster order */
    const uint64_t *cluster_sizes; /* nlist */
    /* Optional exact FP32 refinement (hybrid.cuh:171-178, cpu_refinement.cpp:168-181):
     * when exact_base is set, a candidate's distance is the exact squared L2 distance
     * between the raw query and base row ids[gid] (row pid at exact_base + pid *
     * exact_stride floats), the fp32 rounding of the fp64 fma chain over d ascending;
     * candidates whose pid >= exact_rows, or all of them when exact_dim != dim, are
     * dropped (value NaN: never a result, never below a threshold; still counted). */
    const float *exact_base;
    uint64_t exact_rows, exact_dim, exact_stride;
    /* 0 (default): the reference's 2^ex * ip1 + ip2 refinement; 1: the full-code ipT. */
    int refine_full_code;
    /* 0 (default): ip1 from the integer estimator (KernelType::Bitwise); 1: from the fp16
     * LUT estimator (KernelType::Lut4Bit, the reference's default kernel type). */
    int lut_estimator;
    /* 0 (default): squared L2; 1: inner product (the reference CPU path's METRIC_IP): the
     * additive query term of a probed cluster is g_add = -<q', c'> (fp64 chain in ascending
     * order, rounded once; index/query.hpp:99-108, ivf/ivf.hpp:681-706) instead of the
     * squared distance g; the error term stays sqrt(g); probes stay the nearest by g. */
    int metric;
} cora_oracle_index;

#define CORA_ORACLE_VANGUARD_MIN_KEEP 20
#define CORA_ORACLE_VANGUARD_MAX_KEEP 4096 /* also the largest supported topk */

void cora_oracle_rotate(const cora_oracle_index *ix, const float *q, uint64_t nq, float *qr);
void cora_oracle_query_prep(uint64_t D, uint64_t ex_bits, const float *qr, uint64_t nq,
                            float *sumq, float *k1, float *kb, float *width, int32_t *qint,
                            uint32_t *planes);
float cora_oracle_centroid_dist(const float *qr, const float *c, uint64_t D);
void cora_oracle_probe(const cora_oracle_index *ix, const float *qr, uint64_t nq,
                       uint64_t nprobe, int32_t *probe_ids, float *probe_g);
int32_t cora_oracle_ip_int(const cora_oracle_index *ix, uint64_t gid, const uint32_t *planes);
float cora_oracle_low(const cora_oracle_index *ix, uint64_t gid, float ip1, float g, float k1);
/* The same with separate additive and error terms (g_add; gerr = sqrt(max(g, 0))). */
float cora_oracle_low2(const cora_oracle_index *ix, uint64_t gid, float ip1, float g_add,
                       float gerr, float k1);
/* The inner-product metric's additive term: -(fp32 of the fp64 chain sum_j q'_j c_j). */
float cora_oracle_ip_gadd(const float *qr, const float *c, uint64_t D);
void cora_oracle_decode_ex7(const uint8_t *code, uint64_t D, uint8_t *u);
float cora_oracle_ip_total(const float *qr, const uint32_t *bits, const uint8_t *code,
                           uint64_t D);
float cora_oracle_ex(const cora_oracle_index *ix, uint64_t gid, float ip_total, float g,
                     float kb);
/* binary32 -> binary16, round to nearest (ties to even), and binary16 -> binary32. */
uint16_t cora_oracle_f32_to_f16(float f);
float cora_oracle_f16_to_f32(uint16_t h);
/* LUT estimator tables of one rotated query: lut[g * 16 + p], g < D / 4 (binary16 bits). */
void cora_oracle_query_lut(const float *qr, uint64_t D, uint16_t *lut);
/* LUT estimator ip1 of one vector's 1-bit code words (D / 32 words, dim 32w + b at bit 31 - b). */
float cora_oracle_ip_lut(const uint32_t *words, const uint16_t *lut, uint64_t D);
/* ip2 = <q', u>, u the decoded 7-bit ex code (what ip64_fxu7_avx computes). */
float cora_oracle_ip_ex(const float *qr, const uint8_t *code, uint64_t D);
/* The reference's refinement: (f_add_ex + g) + f_rescale_ex * ((128 * ip1 + ip2) + kb). */
float cora_oracle_ex_split(const cora_oracle_index *ix, uint64_t gid, float ip1, float ip2,
                           float g, float kb);

/* Full search. Outputs are row-major nq x k. thresholds0 may be NULL (FLT_MAX).
 * Optional outputs (NULL to skip): cand_count[nq] (= seeds + main candidates),
 * thresholds1[nq] (threshold after vanguard seeding), probe_ids/probe_g [nq x nprobe],
 * cand_gids[nq x cand_cap] (sorted ascending gids of all candidates, truncated at cap).
 * Returns 0, or -1 on invalid arguments. `threads` > 1 parallelises over queries. */
int cora_oracle_search(const cora_oracle_index *ix, const float *q, uint64_t nq, uint64_t k,
                       uint64_t nprobe, uint64_t vanguard, const float *thresholds0,
                       float *out_dist, uint32_t *out_ids, uint64_t *cand_count,
                       float *thresholds1, int32_t *probe_ids, float *probe_g,
                       uint32_t *cand_gids, uint64_t cand_cap, int threads);

/* One shard's part of a cluster-sharded search (the index holds only the shard's clusters;
 * the others have size 0). Same as cora_oracle_search, plus:
 *   seed_keys_out  [nq x k] (NULL to skip): the shard's k smallest seed keys
 *                  (ord(ex) << 32 | id) with ex < T0, ascending, padded with UINT64_MAX;
 *   thresholds1_in [nq]     (NULL: computed from the shard's own seeds): the threshold of
 *                  the main pass, i.e. min(T0, k-th smallest key over every shard's
 *                  seed_keys_out) when at least k exist, else T0;
 *   topk_keys_out  [nq x k] (NULL to skip): the shard's top-k keys, padded as above.
 * Merging the shards' topk_keys_out (k smallest of the union) gives cora_oracle_search's
 * result on the whole index. */
int cora_oracle_search_shard(const cora_oracle_index *ix, const float *q, uint64_t nq,
                             uint64_t k, uint64_t nprobe, uint64_t vanguard,
                             const float *thresholds0, const float *thresholds1_in,
                             uint64_t *seed_keys_out, uint64_t *topk_keys_out, float *out_dist,
                             uint32_t *out_ids, uint64_t *cand_count, int threads);

#ifdef __cplusplus
}
#endif
#endif
