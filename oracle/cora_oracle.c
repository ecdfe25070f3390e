/*
 * TEST INFRASTRUCTURE ONLY — CPU oracle for the IVF-RaBitQ search hot path.
 * See cora_oracle.h for the contract and the reference lines each step restates.
 * Built with -ffp-contract=off -fno-fast-math so every fp32 operation rounds once.
 */
#include "cora_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* Monotone map float -> uint32 used for every (value, id) ordering in the contract. */
static inline uint32_t ord_f32(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

typedef struct {
    uint64_t key; /* (ord(value) << 32) | id */
    float value;
    float ip1;
    uint32_t gid;
    uint32_t probe;
} entry_t;

static int cmp_entry(const void *a, const void *b) {
    const uint64_t x = ((const entry_t *)a)->key, y = ((const entry_t *)b)->key;
    return (x > y) - (x < y);
}
static int cmp_u32(const void *a, const void *b) {
    const uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return (x > y) - (x < y);
}
static int cmp_u64(const void *a, const void *b) {
    const uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return (x > y) - (x < y);
}

/* hybrid.cu:436-440 (cuBLAS SGEMM q' = q*P) restated with fp64 accumulation in ascending
 * input-dimension order. fp32*fp32 products are exact in fp64, so a fused or unfused
 * multiply-add gives the same bits. */
void cora_oracle_rotate(const cora_oracle_index *ix, const float *q, uint64_t nq, float *qr) {
    const uint64_t dim = ix->dim, D = ix->padded_dim;
    for (uint64_t n = 0; n < nq; ++n)
        for (uint64_t j = 0; j < D; ++j) {
            double acc = 0.0;
            for (uint64_t i = 0; i < dim; ++i)
                acc += (double)q[n * dim + i] * (double)ix->rotator[i * D + j];
            qr[n * D + j] = (float)acc;
        }
}

/* query_kernels.cuh:73-94 (sumq, k1 = -0.5 sumq, kb = -(2^(ex+1)-1)/2 sumq) and
 * query_kernels.cuh:117-189 (width = max(amax/127, 1e-30), qint = clamp(rn(q'/width)),
 * plane j word w bit (31-b) = bit j of qint[32w+b]). sumq accumulates in fp64: lane l of
 * 32 sums dims l, l+32, ... in ascending order, then an xor butterfly (16,8,4,2,1). */
void cora_oracle_query_prep(uint64_t D, uint64_t ex_bits, const float *qr, uint64_t nq,
                            float *sumq, float *k1, float *kb, float *width, int32_t *qint,
                            uint32_t *planes) {
    const uint64_t W = D / 32;
    const float c1 = -0.5f;
    const float cb = -(float)((1u << (ex_bits + 1)) - 1u) / 2.0f;
    for (uint64_t n = 0; n < nq; ++n) {
        const float *x = qr + n * D;
        double part[32], next[32];
        float amax = 0.0f;
        for (int l = 0; l < 32; ++l) {
            double acc = 0.0;
            for (uint64_t j = (uint64_t)l; j < D; j += 32) acc += (double)x[j];
            part[l] = acc;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            for (int l = 0; l < 32; ++l) next[l] = part[l] + part[l ^ off];
            memcpy(part, next, sizeof(part));
        }
        for (uint64_t j = 0; j < D; ++j) amax = fmaxf(amax, fabsf(x[j]));
        const float sf = (float)part[0];
        if (sumq) sumq[n] = sf;
        if (k1) k1[n] = sf * c1;
        if (kb) kb[n] = sf * cb;
        const float w = fmaxf(amax / 127.0f, 1e-30f);
        const float inv = 1.0f / w;
        if (width) width[n] = w;
        uint32_t *pl = planes ? planes + n * 8 * W : NULL;
        if (pl) memset(pl, 0, 8 * W * sizeof(uint32_t));
        for (uint64_t j = 0; j < D; ++j) {
            const float p = x[j] * inv;
            int v = (int)nearbyintf(p); /* round half to even, as __float2int_rn */
            if (v < -128) v = -128;
            if (v > 127) v = 127;
            if (qint) qint[n * D + j] = v;
            if (pl) {
                const uint32_t bits = (uint32_t)v & 0xFFu;
                for (int b = 0; b < 8; ++b)
                    if ((bits >> b) & 1u) pl[b * W + j / 32] |= 1u << (31 - (j % 32));
            }
        }
    }
}

/* g_add = ||q' - c'||^2 (hybrid.cu:465-477 computes ||q||^2+||c||^2-2q.c in fp32; here
 * it is one fp64 fma chain in ascending dimension order, rounded once). */
float cora_oracle_centroid_dist(const float *qr, const float *c, uint64_t D) {
    double acc = 0.0;
    for (uint64_t j = 0; j < D; ++j) {
        const double d = (double)qr[j] - (double)c[j];
        acc = fma(d, d, acc);
    }
    return (float)acc;
}

static void probe_one(const cora_oracle_index *ix, const float *x, uint64_t nprobe,
                      int32_t *pid_out, float *pg_out, entry_t *scratch) {
    const uint64_t D = ix->padded_dim;
    for (uint64_t c = 0; c < ix->nlist; ++c) {
        const float g = cora_oracle_centroid_dist(x, ix->centroids + c * D, D);
        scratch[c].value = g;
        scratch[c].key = ((uint64_t)ord_f32(g) << 32) | (uint32_t)c;
    }
    qsort(scratch, ix->nlist, sizeof(entry_t), cmp_entry);
    for (uint64_t r = 0; r < nprobe; ++r) {
        pid_out[r] = (int32_t)(scratch[r].key & 0xFFFFFFFFu);
        pg_out[r] = scratch[r].value;
    }
}

/* select_k(select_min, sorted) over g_add, hybrid.cu:485-493, ties by cluster id. */
void cora_oracle_probe(const cora_oracle_index *ix, const float *qr, uint64_t nq,
                       uint64_t nprobe, int32_t *probe_ids, float *probe_g) {
    entry_t *scratch = (entry_t *)malloc(ix->nlist * sizeof(entry_t));
    for (uint64_t n = 0; n < nq; ++n)
        probe_one(ix, qr + n * ix->padded_dim, nprobe, probe_ids + n * nprobe,
                  probe_g + n * nprobe, scratch);
    free(scratch);
}

static uint64_t *cluster_starts(const cora_oracle_index *ix) {
    uint64_t *s = (uint64_t *)malloc((ix->nlist + 1) * sizeof(uint64_t));
    s[0] = 0;
    for (uint64_t c = 0; c < ix->nlist; ++c) s[c + 1] = s[c] + ix->cluster_sizes[c];
    return s;
}

static int32_t ip_int_at(const cora_oracle_index *ix, uint64_t start, uint64_t n, uint64_t i,
                         const uint32_t *planes) {
    const uint64_t W = ix->padded_dim / 32;
    int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (uint64_t w = 0; w < W; ++w) {
        const uint32_t x = ix->short_data[start * W + w * n + i];
        for (int j = 0; j < 8; ++j) acc[j] += __builtin_popcount(x & planes[j * W + w]);
    }
    /* filter_kernels.cuh:100-104: the high plane carries weight -2^7 */
    int32_t ip = -(acc[7] << 7);
    for (int j = 0; j < 7; ++j) ip += acc[j] << j;
    return ip;
}

int32_t cora_oracle_ip_int(const cora_oracle_index *ix, uint64_t gid, const uint32_t *planes) {
    uint64_t start = 0, c = 0;
    while (start + ix->cluster_sizes[c] <= gid) start += ix->cluster_sizes[c++];
    return ip_int_at(ix, start, ix->cluster_sizes[c], gid - start, planes);
}

/* filter_kernels.cuh:693-696: low = f_add + g + f_rescale*(ip1 + k1) - f_error*sqrt(g),
 * with sqrt's argument clamped at zero. */
float cora_oracle_low2(const cora_oracle_index *ix, uint64_t gid, float ip1, float g_add,
                       float gerr, float k1) {
    const float *f = ix->short_factors + gid * 3;
    const float a = f[0] + g_add;
    const float b = f[1] * (ip1 + k1);
    const float e = f[2] * gerr;
    return (a + b) - e;
}

float cora_oracle_low(const cora_oracle_index *ix, uint64_t gid, float ip1, float g, float k1) {
    return cora_oracle_low2(ix, gid, ip1, g, sqrtf(fmaxf(g, 0.0f)), k1);
}

/* ivf.hpp:699-706 (dot_product of the rotated query and the centroid) negated, as
 * set_g_add(dist, ip) stores it for METRIC_IP (query.hpp:99-108). */
float cora_oracle_ip_gadd(const float *qr, const float *c, uint64_t D) {
    double acc = 0.0;
    for (uint64_t j = 0; j < D; ++j) acc = fma((double)qr[j], (double)c[j], acc);
    return -(float)acc;
}

/* IEEE 754 binary32 -> binary16 with round to nearest, ties to even (the rounding of
 * CUDA's __float2half_rn, which the reference's table kernel uses), from the format's
 * definition: normal results keep 10 of the 23 fraction bits and round on the 13 dropped
 * ones; results below 2^-14 are multiples of 2^-24 rounded from the full significand;
 * magnitudes from 65520 (half-way between the largest half, 65504, and 2^16) up are inf. */
uint16_t cora_oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 */
    if (ax >= 0x38800000u) {                                  /* >= 2^-14: normal half */
        const uint32_t r = ax - 0x38000000u;                  /* exponent bias 127 -> 15 */
        uint32_t h = r >> 13;
        const uint32_t rest = r & 0x1FFFu;
        if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h; /* a carry may bump the exponent */
        return (uint16_t)(sign | h);
    }
    const uint32_t e = ax >> 23;
    if (e < 102) return sign; /* below 2^-25: rounds to zero */
    const uint32_t m24 = (ax & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e; /* value / 2^-24 = m24 / 2^shift, shift in [14, 24] */
    uint32_t k = m24 >> shift;
    const uint32_t rest = m24 & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
    if (rest > halfway || (rest == halfway && (k & 1u))) ++k; /* k = 1024: the smallest normal */
    return (uint16_t)(sign | k);
}

float cora_oracle_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u;
    uint32_t x;
    if (e == 0) {
        const float v = (float)m * 0x1p-24f; /* exact */
        memcpy(&x, &v, 4);
        x |= sign;
    } else if (e == 31) {
        x = sign | 0x7F800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* query_kernels.cuh:199-221 (precompute_lut_fp16_kernel): entry (g, p) is the fp32 sum,
 * starting from 0, of q'[4g + i] over the bits 3 - i set in p (i ascending), rounded to
 * binary16. */
void cora_oracle_query_lut(const float *qr, uint64_t D, uint16_t *lut) {
    for (uint64_t g = 0; g < D / 4; ++g)
        for (int p = 0; p < 16; ++p) {
            float sum = 0.0f;
            for (int i = 0; i < 4; ++i)
                if (p & (8 >> i)) sum += qr[4 * g + (uint64_t)i];
            lut[g * 16 + (uint64_t)p] = cora_oracle_f32_to_f16(sum);
        }
}

/* filter_kernels.cuh:283-306 / 655-694: nibble n of word w (its dims 32w + 4n ..) adds entry
 * (8w + n, nibble) to acc0 for even n and to acc1 for odd n, in order; ip1 = acc0 + acc1. */
float cora_oracle_ip_lut(const uint32_t *words, const uint16_t *lut, uint64_t D) {
    float acc0 = 0.0f, acc1 = 0.0f;
    for (uint64_t w = 0; w < D / 32; ++w)
        for (int n = 0; n < 8; ++n) {
            const uint32_t nib = (words[w] >> (28 - 4 * n)) & 0xFu;
            const float v = cora_oracle_f16_to_f32(lut[(8 * w + (uint64_t)n) * 16 + nib]);
            if (n & 1)
                acc1 += v;
            else
                acc0 += v;
        }
    return acc0 + acc1;
}

/* Inverse of pack_excode.hpp:216-264 (packing_7bit_excode), per 64 dims = 56 bytes. */
void cora_oracle_decode_ex7(const uint8_t *code, uint64_t D, uint8_t *u) {
    for (uint64_t b = 0; b < D / 64; ++b) {
        const uint8_t *p = code + b * 56;
        uint8_t *o = u + b * 64;
        for (int k = 0; k < 16; ++k) {
            o[k] = p[k] & 63u;
            o[16 + k] = p[16 + k] & 63u;
            o[32 + k] = p[32 + k] & 63u;
            o[48 + k] = (uint8_t)((p[k] >> 6) | ((p[16 + k] >> 6) << 2) | ((p[32 + k] >> 6) << 4));
        }
        uint64_t top = 0;
        for (int t = 0; t < 8; ++t) top |= (uint64_t)p[48 + t] << (8 * t);
        for (int d = 0; d < 64; ++d) o[d] |= (uint8_t)(((top >> (8 * (d % 8) + d / 8)) & 1u) << 6);
    }
}

/* The refinement's fp64 inner product sum_d qr_d * c_d of D integer codes c (c_d < 256),
 * in this engine's fixed summation order: 16-dimension chunks (chunk k = dims 16k .. 16k + 15),
 * partial sum j over the chunks k with k % 8 == j (chunks ascending, dims ascending in a
 * chunk; every product is exact in fp64), combined as ((p0 + p1) + (p2 + p3)) +
 * ((p4 + p5) + (p6 + p7)), rounded once to fp32. The reference (ip64_fxu7_avx,
 * utils/space.hpp:677-762) sums in its own fp32 SIMD order; the two agree to rounding. */
static float refine_dot(const float *qr, const uint8_t *c, uint64_t D) {
    double p[8] = {0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0};
    for (uint64_t d = 0; d < D; ++d) p[(d / 16) % 8] += (double)qr[d] * (double)c[d];
    const double a = (p[0] + p[1]) + (p[2] + p[3]);
    const double b = (p[4] + p[5]) + (p[6] + p[7]);
    return (float)(a + b);
}

/* Refinement inner product of the full (1 + ex_bits)-bit code with the rotated query:
 * ipT = sum_d q'_d * (2^ex_bits * b_d + u_d), b the 1-bit code (bit 31-(d%32) of word d/32),
 * u the decoded 7-bit ex code. The reference forms the same quantity as
 * 2^ex_bits * ip1 + ip2 (cpu_refinement.cpp:183-191) with ip1 taken from its fp16-LUT or
 * 8-bit-query scan; here it is one fp64 sum (refine_dot's order), rounded once to fp32. */
float cora_oracle_ip_total(const float *qr, const uint32_t *bits, const uint8_t *code,
                           uint64_t D) {
    uint8_t u[4096];
    cora_oracle_decode_ex7(code, D, u);
    for (uint64_t d = 0; d < D; ++d) {
        const uint32_t bit = (bits[d / 32] >> (31 - (d % 32))) & 1u;
        u[d] = (uint8_t)(128u * bit + u[d]);
    }
    return refine_dot(qr, u, D);
}

/* Full-code form (opt-in): ex = (f_add_ex + g) + f_rescale_ex * (ipT + kb), ipT the
 * full-code inner product above in place of the reference's 2^ex_bits * ip1 + ip2. */
float cora_oracle_ex(const cora_oracle_index *ix, uint64_t gid, float ip_total, float g,
                     float kb) {
    const float *f = ix->ex_factors + gid * 2;
    return (f[0] + g) + (f[1] * (ip_total + kb));
}

/* ip2 of cpu_refinement.cpp:183-185: <q', u> over the decoded 7-bit ex code, the quantity
 * ip64_fxu7_avx (utils/space.hpp:677-762) computes; here one fp64 sum in refine_dot's order
 * (products exact), rounded once. */
float cora_oracle_ip_ex(const float *qr, const uint8_t *code, uint64_t D) {
    uint8_t u[4096];
    cora_oracle_decode_ex7(code, D, u);
    return refine_dot(qr, u, D);
}

/* cpu_refinement.cpp:186-191 (= split_distance_boosting, estimator.hpp:86-103):
 * ex = (f_add_ex + g) + f_rescale_ex * ((2^ex_bits * ip1 + ip2) + kb), evaluated in that
 * order in fp32 (2^7 * ip1 is exact). */
float cora_oracle_ex_split(const cora_oracle_index *ix, uint64_t gid, float ip1, float ip2,
                           float g, float kb) {
    const float *f = ix->ex_factors + gid * 2;
    const float t = ((128.0f * ip1) + ip2) + kb;
    return (f[0] + g) + (f[1] * t);
}

static void vector_bits(const cora_oracle_index *ix, uint64_t start, uint64_t n, uint64_t i,
                        uint32_t *out) {
    const uint64_t W = ix->padded_dim / 32;
    for (uint64_t w = 0; w < W; ++w) out[w] = ix->short_data[start * W + w * n + i];
}

/* Exact FP32 refinement of gid against the raw query qraw (see cora_oracle_index). */
static float exact_refine(const cora_oracle_index *ix, const float *qraw, uint64_t gid) {
    const uint64_t pid = ix->ids[gid];
    if (ix->exact_dim != ix->dim || pid >= ix->exact_rows) return NAN;
    const float *b = ix->exact_base + pid * ix->exact_stride;
    double acc = 0.0;
    for (uint64_t d = 0; d < ix->dim; ++d) {
        const double diff = (double)qraw[d] - (double)b[d];
        acc = fma(diff, diff, acc);
    }
    return (float)acc;
}

/* Refinement of vector i of the cluster at `start` (size n); ip1 is the scan's estimate. */
static float refine(const cora_oracle_index *ix, const float *qraw, const float *x,
                    uint64_t start, uint64_t n, uint64_t i, float ip1, float g, float kb) {
    uint32_t bits[128];
    const uint64_t D = ix->padded_dim, LC = D * ix->ex_bits / 8, gid = start + i;
    const uint8_t *code = ix->long_codes + gid * LC;
    if (ix->exact_base) return exact_refine(ix, qraw, gid);
    if (!ix->refine_full_code)
        return cora_oracle_ex_split(ix, gid, ip1, cora_oracle_ip_ex(x, code, D), g, kb);
    vector_bits(ix, start, n, i, bits);
    return cora_oracle_ex(ix, gid, cora_oracle_ip_total(x, bits, code, D), g, kb);
}

/* The scan's ip1 of vector i of the cluster at `start` (size n): the integer estimator's
 * width * ip_int (+ 0, filter_kernels.cuh:106), or the LUT estimator's sum (lut != NULL). */
static float scan_ip1(const cora_oracle_index *ix, uint64_t start, uint64_t n, uint64_t i,
                      const uint32_t *planes, float width, const uint16_t *lut) {
    if (lut) {
        uint32_t words[128];
        vector_bits(ix, start, n, i, words);
        return cora_oracle_ip_lut(words, lut, ix->padded_dim);
    }
    return width * (float)ip_int_at(ix, start, n, i, planes) + 0.0f;
}

static void push(entry_t **v, uint64_t *n, uint64_t *cap, entry_t e) {
    if (*n == *cap) {
        *cap = *cap ? *cap * 2 : 256;
        *v = (entry_t *)realloc(*v, *cap * sizeof(entry_t));
    }
    (*v)[(*n)++] = e;
}

/* k smallest keys of res[] with value < T0, ascending, padded with UINT64_MAX. */
static void smallest_keys(const entry_t *res, uint64_t nres, float T0, uint64_t k,
                          uint64_t *out) {
    uint64_t *tmp = (uint64_t *)malloc((nres ? nres : 1) * sizeof(uint64_t));
    uint64_t m = 0;
    for (uint64_t i = 0; i < nres; ++i)
        if (res[i].value < T0) tmp[m++] = res[i].key;
    qsort(tmp, m, sizeof(uint64_t), cmp_u64);
    for (uint64_t i = 0; i < k; ++i) out[i] = i < m ? tmp[i] : UINT64_MAX;
    free(tmp);
}

static int search_impl(const cora_oracle_index *ix, const float *q, uint64_t nq, uint64_t k,
                       uint64_t nprobe, uint64_t vanguard, const float *thresholds0,
                       float *out_dist, uint32_t *out_ids, uint64_t *cand_count,
                       float *thresholds1, int32_t *probe_ids_out, float *probe_g_out,
                       uint32_t *cand_gids, uint64_t cand_cap, int threads,
                       const float *thresholds1_in, uint64_t *seed_keys_out,
                       uint64_t *topk_keys_out) {
    if (!ix || !q || !out_dist || !out_ids || k == 0 || k > CORA_ORACLE_VANGUARD_MAX_KEEP ||
        nprobe == 0 || nprobe > ix->nlist ||
        ix->padded_dim % 64 || ix->padded_dim > 4096 || ix->ex_bits != 7)
        return -1;
    const uint64_t D = ix->padded_dim, W = D / 32;
    const uint64_t keep = k > CORA_ORACLE_VANGUARD_MIN_KEEP ? k : CORA_ORACLE_VANGUARD_MIN_KEEP;
    /* Seeding depth: the vanguard size, but at least the nearest probe, so that the
     * static main-phase threshold always prunes (the reference's CPU refiner lowers its
     * thresholds continuously instead, cpu_refinement.cpp:217-228). */
    const uint64_t vdepth = vanguard > 0 ? vanguard : 1;
    const uint64_t veff = vdepth < nprobe ? vdepth : nprobe;
    uint64_t *starts = cluster_starts(ix);
    if (threads < 1) threads = 1;

#pragma omp parallel for schedule(dynamic, 1) num_threads(threads)
    for (int64_t qi = 0; qi < (int64_t)nq; ++qi) {
        const uint64_t n = (uint64_t)qi;
        float *x = (float *)malloc(D * sizeof(float));
        uint32_t *planes = (uint32_t *)malloc(8 * W * sizeof(uint32_t));
        entry_t *scratch = (entry_t *)malloc(ix->nlist * sizeof(entry_t));
        int32_t *pid = (int32_t *)malloc(nprobe * sizeof(int32_t));
        float *pg = (float *)malloc(nprobe * sizeof(float));
        entry_t *res = NULL, *pair = NULL;
        uint64_t nres = 0, cres = 0, npair = 0, cpair = 0;
        float sumq, k1, kb, width;
        uint16_t *lut = ix->lut_estimator ? (uint16_t *)malloc(4 * D * sizeof(uint16_t)) : NULL;

        cora_oracle_rotate(ix, q + n * ix->dim, 1, x);
        cora_oracle_query_prep(D, ix->ex_bits, x, 1, &sumq, &k1, &kb, &width, NULL, planes);
        if (lut) cora_oracle_query_lut(x, D, lut);
        probe_one(ix, x, nprobe, pid, pg, scratch);
        if (probe_ids_out) memcpy(probe_ids_out + n * nprobe, pid, nprobe * sizeof(int32_t));
        if (probe_g_out) memcpy(probe_g_out + n * nprobe, pg, nprobe * sizeof(float));
        /* the additive term of each probe (the squared distance for L2) */
        float *pga = (float *)malloc(nprobe * sizeof(float));
        for (uint64_t r = 0; r < nprobe; ++r)
            pga[r] = ix->metric == 1 ? cora_oracle_ip_gadd(x, ix->centroids + (uint64_t)pid[r] * D, D)
                                     : pg[r];

        const float T0 = thresholds0 ? thresholds0[n] : FLT_MAX;
        uint64_t *bound = (uint64_t *)malloc((veff ? veff : 1) * sizeof(uint64_t));
        int *take_all = (int *)malloc((veff ? veff : 1) * sizeof(int));

        /* Vanguard: the first veff probes keep their top max(k,20) by (low, gid) among
         * low < T0 as seeds (filter_kernels.cuh:308-468), refined right away. */
        for (uint64_t r = 0; r < veff; ++r) {
            const uint64_t c = (uint64_t)pid[r], s = starts[c], nc = ix->cluster_sizes[c];
            const float g = pga[r], gerr = sqrtf(fmaxf(pg[r], 0.0f));
            npair = 0;
            for (uint64_t i = 0; i < nc; ++i) {
                const float ip1 = scan_ip1(ix, s, nc, i, planes, width, lut);
                const float low = cora_oracle_low2(ix, s + i, ip1, g, gerr, k1);
                if (low < T0) {
                    entry_t e = {((uint64_t)ord_f32(low) << 32) | (uint32_t)(s + i), low, ip1,
                                 (uint32_t)(s + i), (uint32_t)r};
                    push(&pair, &npair, &cpair, e);
                }
            }
            qsort(pair, npair, sizeof(entry_t), cmp_entry);
            take_all[r] = npair <= keep;
            bound[r] = take_all[r] ? 0 : pair[keep - 1].key;
            const uint64_t ns = take_all[r] ? npair : keep;
            for (uint64_t i = 0; i < ns; ++i) {
                const uint32_t gid = pair[i].gid;
                const float ex = refine(ix, q + n * ix->dim, x, s, nc, gid - s, pair[i].ip1, g, kb);
                entry_t e = {((uint64_t)ord_f32(ex) << 32) | ix->ids[gid], ex, pair[i].ip1, gid,
                             (uint32_t)r};
                push(&res, &nres, &cres, e);
            }
        }
        /* T1 = k-th smallest seed distance below T0, when at least k exist (over every
         * shard's seeds when the caller passes it in). */
        if (seed_keys_out) smallest_keys(res, nres, T0, k, seed_keys_out + n * k);
        float T1 = T0;
        if (thresholds1_in) {
            T1 = thresholds1_in[n];
        } else {
            uint64_t nv = 0;
            for (uint64_t i = 0; i < nres; ++i)
                if (res[i].value < T0) ++nv;
            if (nv >= k) {
                entry_t *tmp = (entry_t *)malloc(nv * sizeof(entry_t));
                uint64_t m = 0;
                for (uint64_t i = 0; i < nres; ++i)
                    if (res[i].value < T0) tmp[m++] = res[i];
                qsort(tmp, nv, sizeof(entry_t), cmp_entry);
                T1 = tmp[k - 1].value;
                free(tmp);
            }
        }
        if (thresholds1) thresholds1[n] = T1;

        /* Main scan over every probe against the static T1; vanguard probes skip their
         * seeds (keys at or below the recorded boundary). */
        for (uint64_t r = 0; r < nprobe; ++r) {
            const uint64_t c = (uint64_t)pid[r], s = starts[c], nc = ix->cluster_sizes[c];
            const float g = pga[r], gerr = sqrtf(fmaxf(pg[r], 0.0f));
            if (r < veff && take_all[r]) continue;
            for (uint64_t i = 0; i < nc; ++i) {
                const float ip1 = scan_ip1(ix, s, nc, i, planes, width, lut);
                const float low = cora_oracle_low2(ix, s + i, ip1, g, gerr, k1);
                if (!(low < T1)) continue;
                if (r < veff) {
                    const uint64_t key = ((uint64_t)ord_f32(low) << 32) | (uint32_t)(s + i);
                    if (key <= bound[r]) continue;
                }
                const uint32_t gid = (uint32_t)(s + i);
                const float ex = refine(ix, q + n * ix->dim, x, s, nc, i, ip1, g, kb);
                entry_t e = {((uint64_t)ord_f32(ex) << 32) | ix->ids[gid], ex, ip1, gid,
                             (uint32_t)r};
                push(&res, &nres, &cres, e);
            }
        }
        if (cand_count) cand_count[n] = nres;
        if (cand_gids && cand_cap) {
            uint32_t *g = cand_gids + n * cand_cap;
            const uint64_t m = nres < cand_cap ? nres : cand_cap;
            uint32_t *all = (uint32_t *)malloc((nres ? nres : 1) * sizeof(uint32_t));
            for (uint64_t i = 0; i < nres; ++i) all[i] = res[i].gid;
            qsort(all, nres, sizeof(uint32_t), cmp_u32);
            for (uint64_t i = 0; i < cand_cap; ++i) g[i] = i < m ? all[i] : 0xFFFFFFFFu;
            free(all);
        }
        /* Output: ascending (ex, id) among ex < T0, padded with (FLT_MAX, 0)
         * (cpu_refinement.cpp:197-230,269-283). */
        qsort(res, nres, sizeof(entry_t), cmp_entry);
        if (topk_keys_out) smallest_keys(res, nres, T0, k, topk_keys_out + n * k);
        uint64_t o = 0;
        for (uint64_t i = 0; i < nres && o < k; ++i) {
            if (!(res[i].value < T0)) continue;
            out_dist[n * k + o] = res[i].value;
            out_ids[n * k + o] = (uint32_t)(res[i].key & 0xFFFFFFFFu);
            ++o;
        }
        for (; o < k; ++o) {
            out_dist[n * k + o] = FLT_MAX;
            out_ids[n * k + o] = 0;
        }
        free(x); free(planes); free(scratch); free(pid); free(pg); free(res); free(pair);
        free(bound); free(take_all); free(lut); free(pga);
    }
    free(starts);
    return 0;
}

int cora_oracle_search(const cora_oracle_index *ix, const float *q, uint64_t nq, uint64_t k,
                       uint64_t nprobe, uint64_t vanguard, const float *thresholds0,
                       float *out_dist, uint32_t *out_ids, uint64_t *cand_count,
                       float *thresholds1, int32_t *probe_ids_out, float *probe_g_out,
                       uint32_t *cand_gids, uint64_t cand_cap, int threads) {
    return search_impl(ix, q, nq, k, nprobe, vanguard, thresholds0, out_dist, out_ids,
                       cand_count, thresholds1, probe_ids_out, probe_g_out, cand_gids, cand_cap,
                       threads, NULL, NULL, NULL);
}

int cora_oracle_search_shard(const cora_oracle_index *ix, const float *q, uint64_t nq,
                             uint64_t k, uint64_t nprobe, uint64_t vanguard,
                             const float *thresholds0, const float *thresholds1_in,
                             uint64_t *seed_keys_out, uint64_t *topk_keys_out, float *out_dist,
                             uint32_t *out_ids, uint64_t *cand_count, int threads) {
    return search_impl(ix, q, nq, k, nprobe, vanguard, thresholds0, out_dist, out_ids,
                       cand_count, NULL, NULL, NULL, NULL, 0, threads, thresholds1_in,
                       seed_keys_out, topk_keys_out);
}
