// B200-native IVF-RaBitQ search engine: host orchestration and the C ABI of
// include/cora_b200.h. One engine owns one GPU's copy (or shard) of an index, its
// workspace and one CUDA stream; every search is a fixed sequence of kernels on that
// stream with no host round trip until the results are read back.
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/cora_b200.h"
#include "common.cuh"
#include "kernels_probe.cuh"
#include "kernels_query.cuh"
#include "kernels_refine.cuh"
#include "kernels_scan.cuh"

namespace cora {
namespace {

thread_local std::string g_last_error;

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string &m) : std::runtime_error(m), code(c) {}
};
[[noreturn]] void fail(int code, const std::string &msg) { throw Error(code, msg); }

#define CUDA_TRY(call)                                                                  \
    do {                                                                                \
        cudaError_t e_ = (call);                                                        \
        if (e_ != cudaSuccess)                                                          \
            ::cora::fail(CORA_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// Limits of the reference (include/coraanns/search/parameters.hpp:9-13).
constexpr uint64_t kDefaultVanguard = 5, kMaxQueryChunk = 65535, kMaxProbeCount = 65536;
constexpr uint64_t kDefaultQueueCapacity = 1ull << 26, kDefaultSpillCapacity = 1ull << 24;
constexpr uint64_t kMaxTopk = 4096, kMaxProbeFast = 4096, kMaxPaddedDim = 1024;
constexpr int kVanguardMinKeep = 20;
constexpr uint32_t kMaxShards = 256;

// parameters.hpp:15-25
void validate_search_shape(uint64_t queries, uint64_t topk, uint64_t nprobe, uint64_t centroids,
                           uint64_t padded_dim) {
    if (queries == 0 || queries > kMaxQueryChunk)
        fail(CORA_EINVAL, "query count must be in [1, 65535]; split larger batches");
    if (topk == 0 || topk > INT_MAX / queries)
        fail(CORA_EINVAL, "topk must be positive and queries * topk must fit an int");
    if (nprobe == 0 || nprobe > kMaxProbeCount || nprobe > centroids)
        fail(CORA_EINVAL, "nprobe must be in [1, min(nlist, 65536)]");
    if (centroids > INT_MAX / queries || padded_dim == 0 || padded_dim > INT_MAX / (queries * 4))
        fail(CORA_EINVAL, "query workspace exceeds kernel indexing limits");
}

template <typename T>
struct DevBuf {
    T *p = nullptr;
    size_t n = 0;
    void alloc(size_t count) {
        release();
        if (count == 0) return;
        CUDA_TRY(cudaMalloc(&p, count * sizeof(T)));
        n = count;
    }
    void release() noexcept {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    ~DevBuf() { release(); }
};

}  // namespace

enum class ScanPhase { kRescanVanguard, kWriteLows, kMain };

struct ScanLaunch {
    IndexView ix;
    SearchView sv;
    int rescan_sort_n;
    uint64_t n_van;
    const ScanItem *items;
    const uint32_t *n_items;
    const uint32_t *pairs;
    int *item_counter;
    const uint8_t *owned;
    int num_sms;
    cudaStream_t st;
};

// ---- tensor maps for the probe GEMM (driver entry point, no libcuda link) ----------------
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) fail(CORA_ECUDA, "the driver does not provide cuTensorMapEncodeTiled");
    return fn;
}

// 2-D fp32 tensor map over `rows` rows of `cols` floats, `ld` floats apart (ld % 4 == 0,
// 16-byte aligned base); box of box_cols x box_rows with 128-byte swizzle (box_cols * 4 <=
// 128); reads past the edges return zeros, stores past them are dropped.
inline CUtensorMap map_f32_2d(const float *base, uint64_t cols, uint64_t rows, uint64_t ld,
                              uint32_t box_cols, uint32_t box_rows) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 4};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_tiled()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                                      const_cast<float *>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        fail(CORA_ECUDA, "cuTensorMapEncodeTiled failed with status " + std::to_string(int(r)));
    return m;
}

inline uint64_t approx_ld(uint64_t nlist) { return (nlist + 3) & ~uint64_t(3); }

// Centroid matrices above this size are multiplied in query-block-fastest tile order (see
// probe_gemm_kernel).
constexpr uint64_t kPgQueryFastBytes = 32ull << 20;

// approx[q * ld + c] = ||q'||^2 + ||c||^2 - 2 <q', c> for every query and centroid, on the
// tensor cores (probe_gemm_kernel; persistent, one CTA per SM at most).
inline void launch_probe_gemm(const float *qr, const float *qnorm2, uint64_t nq, uint64_t D,
                              const float *cent, const float *cnorm2, uint64_t nlist,
                              float *approx, float *chunk_min, int num_sms, cudaStream_t st,
                              int *err) {
    const CUtensorMap tq = map_f32_2d(qr, D, nq, D, kPgBK, kPgBM);
    const CUtensorMap tc = map_f32_2d(cent, D, nlist, D, kPgBK, kPgBN);
    const CUtensorMap to = map_f32_2d(approx, nlist, nq, approx_ld(nlist), 32, kPgBM);
    const size_t sm = probe_gemm_smem();
    CUDA_TRY(cudaFuncSetAttribute(probe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sm));
    const uint64_t tiles = ((nq + kPgBM - 1) / kPgBM) * ((nlist + kPgBN - 1) / kPgBN);
    const unsigned grid = static_cast<unsigned>(std::min<uint64_t>(tiles, (uint64_t)num_sms));
    const int qfast = nlist * D * sizeof(float) > kPgQueryFastBytes ? 1 : 0;
    probe_gemm_kernel<<<grid, kPgThreads, sm, st>>>(tq, tc, to, qnorm2, cnorm2,
                                                    static_cast<int>(nq), static_cast<int>(nlist),
                                                    static_cast<int>(D), chunk_min, qfast, err);
    CUDA_TRY(cudaGetLastError());
}

// Exact top-nprobe from the approximate distances: one warp per query when nprobe <= 32
// (queries whose candidate set overflows go on to the block kernel through `fallback`,
// 1 + nq words), else one CTA per query.
// rotate_prep_kernel with kRotQueriesWide queries per CTA when D <= 128, else kRotQueries.
inline void launch_rotate_prep(const float *raw_q, uint64_t nq, uint64_t dim, uint64_t D, int W4,
                               const double *rotator, float c_b, float *qr, QueryScalars *scal,
                               uint32_t *planes, float *qnorm2, float *ipm, cudaStream_t st) {
    const bool wide = D <= 128;
    const int qpc = wide ? kRotQueriesWide : kRotQueries;
    const size_t sm = (size_t)qpc * (2 * dim + D) * 4;
    const unsigned grid = static_cast<unsigned>((nq + qpc - 1) / qpc);
    const int inq = static_cast<int>(nq), idim = static_cast<int>(dim), iD = static_cast<int>(D);
    if (wide) {
        CUDA_TRY(cudaFuncSetAttribute(rotate_prep_kernel<kRotQueriesWide>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        rotate_prep_kernel<kRotQueriesWide><<<grid, 256, sm, st>>>(
            raw_q, inq, idim, iD, W4, rotator, c_b, qr, scal, planes, qnorm2, ipm);
    } else {
        CUDA_TRY(cudaFuncSetAttribute(rotate_prep_kernel<kRotQueries>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        rotate_prep_kernel<kRotQueries><<<grid, 256, sm, st>>>(
            raw_q, inq, idim, iD, W4, rotator, c_b, qr, scal, planes, qnorm2, ipm);
    }
    CUDA_TRY(cudaGetLastError());
}

inline void launch_guarded_select(float *approx, const float *chunk_min, uint64_t nlist,
                                  uint64_t nq, uint64_t nprobe, const float *qr,
                                  const float *qnorm2, const float *cent, float cmax, uint64_t D,
                                  int *probe_ids, float *probe_g, uint32_t *fallback, int num_sms,
                                  cudaStream_t st) {
    const int inq = static_cast<int>(nq), inp = static_cast<int>(nprobe), iD = static_cast<int>(D);
    const int ccap = guarded_select_cap(inp);
    const size_t bsm = guarded_select_smem(inp, ccap, iD);
    CUDA_TRY(cudaFuncSetAttribute(guarded_select_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm));
    if (nprobe <= 32) {
        const size_t wsm = guarded_select_warp_smem(iD);
        CUDA_TRY(cudaFuncSetAttribute(guarded_select_warp_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsm));
        CUDA_TRY(cudaMemsetAsync(fallback, 0, 4, st));
        guarded_select_warp_kernel<<<static_cast<unsigned>((nq + kGuardWarps - 1) / kGuardWarps),
                                     32 * kGuardWarps, wsm, st>>>(
            approx, chunk_min, static_cast<int>(nlist), approx_ld(nlist), inq, inp, qr, qnorm2,
            cent, cmax, iD, kApproxEpsTF32, probe_ids, probe_g, fallback);
        CUDA_TRY(cudaGetLastError());
        guarded_select_kernel<<<static_cast<unsigned>(2 * num_sms), 256, bsm, st>>>(
            approx, chunk_min, static_cast<int>(nlist), approx_ld(nlist), inp, ccap, qr, qnorm2,
            cent, cmax, iD, kApproxEpsTF32, probe_ids, probe_g, fallback);
    } else {
        guarded_select_kernel<<<inq, 256, bsm, st>>>(approx, chunk_min, static_cast<int>(nlist),
                                                     approx_ld(nlist), inp, ccap, qr, qnorm2, cent,
                                                     cmax, iD, kApproxEpsTF32, probe_ids, probe_g,
                                                     nullptr);
    }
    CUDA_TRY(cudaGetLastError());
}

// refine_kernel instantiation for rows of D bytes and `lanes` lanes per row (8 needs D % 128
// == 0): kC, the chunks a lane loads per round, is its chunk count D / (16 lanes) rounded up
// to one of 1, 2, 4, 6, 8 (with one lane per row kRefineRowChunks: 4, half of the eight
// partials per round, or 8; rows longer than kC chunks per lane take several rounds).
// at most this many chunks per lane and round (measured at D = 768 with 4 lanes, cfg4s:
// candidates 0.795 / 0.903 / 0.850 ms with rounds of 4 / 6 / 8 chunks)
#ifndef CORA_REFINE_KC_MAX
#define CORA_REFINE_KC_MAX 4
#endif
template <int kForm>
RefineKernelFn pick_refine(int D, int lanes) {
    const int nl = std::min(D / (16 * lanes), CORA_REFINE_KC_MAX);
    if (lanes == 1) return kRefineRowChunks == 4 ? refine_kernel<1, 4, kForm> : refine_kernel<1, 8, kForm>;
    if (lanes == 8) {
        if (nl <= 1) return refine_kernel<8, 1, kForm>;
        if (nl <= 2) return refine_kernel<8, 2, kForm>;
        if (nl <= 4) return refine_kernel<8, 4, kForm>;
        if (nl <= 6) return refine_kernel<8, 6, kForm>;
        return refine_kernel<8, 8, kForm>;
    }
    if (nl <= 2) return refine_kernel<4, 2, kForm>;
    if (nl <= 4) return refine_kernel<4, 4, kForm>;
    if (nl <= 6) return refine_kernel<4, 6, kForm>;
    return refine_kernel<4, 8, kForm>;
}

// Lanes per refine row: 1 or 4 when asked for, 8 when asked for and D % 128 == 0 (else 4);
// by default 4 for rows longer than 128 bytes and 1 otherwise (measured at D = 768, cfg4s:
// candidates 0.80 / 0.93 / 0.88 ms with 4 / 1 / 8 lanes; at D = 128, config 2: 0.283 /
// 0.235 / 0.399 ms).
inline int refine_lanes_for(int D, int want) {
    if (want == 8) return D % 128 == 0 ? 8 : 4;
    if (want == 4 || want == 1) return want;
    return D > 128 ? 4 : 1;
}

// One query per CTA: the exact refinement (thread per candidate) when an exact base is set,
// else the lane-shared refine_kernel of the search's refinement form.
inline void launch_refine(const IndexView &ix, const SearchView &sv, int D, int np, int mode,
                          int nq, int lanes_want, cudaStream_t st) {
    const size_t sm = refine_smem(D, np);
    RefineKernelFn kern;
    if (ix.exact_base) {
        kern = refine_exact_kernel;
    } else {
        const int lanes = refine_lanes_for(D, lanes_want);
        if (sv.refine_full_code)
            kern = pick_refine<kRefineFullCode>(D, lanes);
        else if (sv.lut_mode)
            kern = pick_refine<kRefineSplitLut>(D, lanes);
        else
            kern = pick_refine<kRefineSplitInt>(D, lanes);
    }
    CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    kern<<<static_cast<unsigned>(nq), kRefineThreads, sm, st>>>(ix, sv, mode);
    CUDA_TRY(cudaGetLastError());
}

// Cluster-to-shard plan: longest-processing-time greedy on cluster sizes (every vector of an
// index costs the same bytes), largest cluster first (ties: lower cluster id) onto the least
// loaded shard (ties: lower rank). Deterministic, so every rank derives the same plan.
inline void plan_shards(const uint64_t *sizes, uint64_t nlist, uint32_t world, int32_t *owner) {
    std::vector<uint32_t> order(nlist);
    for (uint64_t c = 0; c < nlist; ++c) order[c] = static_cast<uint32_t>(c);
    std::stable_sort(order.begin(), order.end(),
                     [&](uint32_t a, uint32_t b) { return sizes[a] > sizes[b]; });
    std::vector<uint64_t> load(world, 0);
    for (uint32_t c : order) {
        uint32_t best = 0;
        for (uint32_t r = 1; r < world; ++r)
            if (load[r] < load[best]) best = r;
        owner[c] = static_cast<int32_t>(best);
        load[best] += sizes[c];
    }
}

struct Engine {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t last_stream = nullptr;
    cudaEvent_t ev_filter0 = nullptr, ev_filter1 = nullptr;
    // Stage boundary events: a ring of kRing event sets so that timing many back-to-back
    // searches never makes the host wait; a set is read back when it is reused.
    static constexpr int kStages = 13, kRing = 16;
    cudaEvent_t ev_stage[kRing][kStages + 1] = {};
    int ring_next = 0, ring_used = 0, ring_last = -1;
    double stage_sum[kStages] = {};
    uint64_t stage_count = 0;
    int num_sms = 148;

    // index
    bool loaded = false;
    uint64_t N = 0, dim = 0, D = 0, nlist = 0, ex_bits = 0, max_cluster = 0;
    int G16 = 0, W4 = 0, LC = 0;
    DevBuf<float> centroids, cnorm2;  // cnorm2: ||c'||^2 per centroid
    DevBuf<double> rotator;            // dim x D, held in fp64 for the rotation chains
    float cmax = 0.0f;                          // max ||c'|| (rounded up)
    DevBuf<uint4> scan4;
    DevBuf<uint4> rows, meta;  // refine rows (N x D bytes) and meta words (see IndexView)
    std::vector<uint32_t> h_ids;  // original id of every loaded vector (exact refinement)
    // exact FP32 refinement (hybrid.cuh:171-178): the caller's base, borrowed like the
    // reference's mapping, and its rows gathered into HBM in this engine's vector order
    const uint8_t *xb_map = nullptr;
    uint64_t xb_rows = 0, xb_dim = 0, xb_stride = 0, xb_offset = 0;
    DevBuf<float> exact_base;
    DevBuf<uint8_t> exact_ok;
    DevBuf<uint32_t> cl_start, cl_size;
    DevBuf<uint32_t> cl_chunk;              // first 32-vector chunk of each cluster (nlist + 1)
    DevBuf<float4> chunk_range, cl_range;   // factor ranges per chunk / per cluster
    DevBuf<uint8_t> owned;  // optional shard ownership mask (all clusters when empty)

    // options (hybrid.cuh:66-113)
    uint64_t vanguard = kDefaultVanguard;
    uint64_t queue_capacity = kDefaultQueueCapacity, spill_capacity = kDefaultSpillCapacity;
    bool profiling = false, candidate_stats = false, gpu_filter_timing = false;
    bool search_graphs = true;  // replay whole searches from a captured CUDA graph
    bool cross_query_reuse = true, cpu_secondary_filter = true;
    // refinement form: false (default) the reference's 128 ip1 + ip2, true <q', 128 b + u>
    bool refine_full_code = false;
    // estimator of the scan (hybrid.cuh:12 KernelType): 0 Lut4Bit (the fp16-LUT estimator,
    // the reference's default), 1 Bitwise (the integer estimator, this engine's default)
    int ip_kernel_type = 1;
    bool lut_mode() const { return ip_kernel_type == 0; }
    // distance (MetricType of ivf.hpp, defines.hpp:65): 0 squared L2, 1 inner product
    // (distances 1 - <q, x> as estimated by the reference's IP factors); set by the index
    // file, or by cora_set_metric for indexes loaded from raw arrays
    int metric = 0;
    // Upper bound on the HBM buffer holding the vanguard pairs' lower bounds; larger
    // worst cases fall back to rescanning the vanguard clusters.
    uint64_t lows_budget = 16ull << 30;
    int warp_select_limit = kWarpSelectBuf;  // see vanguard_select_warp_kernel
    int topk_warp_limit = kWarpTopBuf;       // see topk_warp_kernel
    int refine_lanes = 0;                    // lanes per refine row: 0 default, 1, 4, 8

    // workspace
    bool ws_ready = false;
    uint64_t ws_q = 0, ws_k = 0, ws_np = 0, ws_vg = 0, cap = 0;
    DevBuf<float> raw_q, qr, qnorm2, gmat, cmin, probe_g, probe_ga, T0, T1, Tcap, out_d;
    DevBuf<QueryScalars> scal;
    DevBuf<float> ipm;   // per query: bound on |fl(ip1 + k1)| for the pruning test
    DevBuf<__half> lut;  // per query: LUT estimator tables (D / 4 groups x 16)
    DevBuf<uint32_t> planes, cand_cnt, seed_cnt, pair_cnt, pair_off, pair_cur, item_off, pairs,
        n_items, out_i;
    DevBuf<int> probe_ids, item_counter, err;
    DevBuf<uint32_t> select_fallback;  // [0] count, [1..] vanguard pairs for block selection
    DevBuf<uint32_t> filt_list;        // [0] count, [1..] vanguard pairs the lows filter reads
    DevBuf<uint64_t> bound, cand_rec, cand_key, vg_off;
    DevBuf<unsigned long long> lows_top;
    DevBuf<float> lows;
    std::vector<uint32_t> h_sizes_sorted;  // cluster sizes, descending (lows worst case)
    DevBuf<ScanItem> items;
    DevBuf<unsigned long long> stats;
    std::vector<float> h_T0;  // host mirror kept for capture/seed without device syncs

    // last-search state
    uint64_t last_nq = 0, last_k = 0, last_np = 0, last_submitted = 0, last_refined = 0;
    const float *last_dq = nullptr;  // device queries of the search in progress

    // cluster sharding (set before loading): this engine keeps the clusters plan_shards()
    // gives `shard_rank` of `shard_world`; split_phase tracks a sharded search in progress
    // (0 none, 1 after begin, 2 after resume).
    uint32_t shard_rank = 0, shard_world = 1;
    uint64_t shard_clusters = 0;
    int split_phase = 0;
    float last_filter_ms = 0.0f;

    // ---- CUDA graph of a whole search (search_host / search_device) ----------------------
    // A search is ~30 dependent launches plus their host-side set-up (function attributes,
    // tensor-map encoding); replaying a captured graph costs one launch. The graph is
    // rebuilt when anything it baked in changes: buffers, shape, stream, or configuration
    // (ws_gen counts loads and workspace changes).
    struct GraphKey {
        const float *d_q = nullptr;
        uint64_t nq = 0, k = 0, np = 0, ws_gen = 0, vanguard = 0;
        float *d_od = nullptr;
        uint32_t *d_oi = nullptr;
        cudaStream_t st = nullptr;
        int wsl = 0, twl = 0, rl = 0;
        bool reuse = false, full_code = false, lut = false;
        int metric = 0;
        bool same(const GraphKey &o) const {
            return d_q == o.d_q && nq == o.nq && k == o.k && np == o.np && ws_gen == o.ws_gen &&
                   vanguard == o.vanguard && d_od == o.d_od && d_oi == o.d_oi && st == o.st &&
                   wsl == o.wsl && twl == o.twl && rl == o.rl && reuse == o.reuse &&
                   full_code == o.full_code && lut == o.lut && metric == o.metric;
        }
    };
    GraphKey graph_key;
    cudaGraphExec_t graph_exec = nullptr;
    uint64_t ws_gen = 0;
    void drop_graph() noexcept {
        if (graph_exec) cudaGraphExecDestroy(graph_exec);
        graph_exec = nullptr;
    }

    explicit Engine(int dev) : device(dev) {
        CUDA_TRY(cudaSetDevice(device));
        CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        CUDA_TRY(cudaEventCreate(&ev_filter0));
        CUDA_TRY(cudaEventCreate(&ev_filter1));
        for (auto &set : ev_stage)
            for (auto &ev : set) CUDA_TRY(cudaEventCreate(&ev));
        CUDA_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device));
        last_stream = stream;
    }
    ~Engine() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        drop_graph();
        free_workspace();
        if (ev_filter0) cudaEventDestroy(ev_filter0);
        if (ev_filter1) cudaEventDestroy(ev_filter1);
        for (auto &set : ev_stage)
            for (auto ev : set)
                if (ev) cudaEventDestroy(ev);
        if (stream) cudaStreamDestroy(stream);
    }

    // ---------------------------------------------------------------- loading
    void load(uint64_t num_vecs, uint64_t d, uint64_t p_d, uint64_t n_centroids, uint64_t ex_b,
              const float *h_centroids, const float *h_rotator, const uint32_t *h_short,
              const float *h_short_factors, const uint8_t *h_long, const float *h_exf,
              const uint32_t *h_ids, const uint64_t *h_sizes) {
        if (loaded) fail(CORA_ESTATE, "index already loaded");
        if (!num_vecs || num_vecs > UINT32_MAX || !d || p_d < d || p_d % 64 || !n_centroids ||
            ex_b > 8 || !h_centroids || !h_rotator || !h_short || !h_short_factors || !h_ids ||
            !h_sizes)
            fail(CORA_EINVAL, "invalid index shape or missing index data");
        if (ex_b != 7 || !h_long || !h_exf)
            fail(CORA_EINVAL, "this engine refines with 7-bit extended codes (8-bit RaBitQ); "
                              "ex_bits must be 7 and extended codes present");
        if (p_d > kMaxPaddedDim) fail(CORA_EINVAL, "padded_dim above 1024 is not supported");
        uint64_t count = 0, largest = 0;
        std::vector<uint32_t> starts(n_centroids), sizes(n_centroids);
        for (uint64_t c = 0; c < n_centroids; ++c) {
            if (h_sizes[c] > num_vecs - count) fail(CORA_EINVAL, "cluster sizes exceed index size");
            starts[c] = static_cast<uint32_t>(count);
            sizes[c] = static_cast<uint32_t>(h_sizes[c]);
            count += h_sizes[c];
            largest = std::max<uint64_t>(largest, h_sizes[c]);
        }
        if (count != num_vecs) fail(CORA_EINVAL, "cluster sizes differ from index size");
        h_sizes_sorted = sizes;
        std::sort(h_sizes_sorted.begin(), h_sizes_sorted.end(), std::greater<uint32_t>());
        CUDA_TRY(cudaSetDevice(device));
        N = num_vecs;
        dim = d;
        D = p_d;
        nlist = n_centroids;
        ex_bits = ex_b;
        max_cluster = largest;
        G16 = static_cast<int>((D + 127) / 128);
        W4 = 4 * G16;
        LC = static_cast<int>(D * ex_bits / 8);
        centroids.alloc(nlist * D);
        rotator.alloc(dim * D);
        CUDA_TRY(cudaMemcpy(centroids.p, h_centroids, nlist * D * 4, cudaMemcpyHostToDevice));
        {
            std::vector<float> cn(nlist);
            double mx = 0.0;
            for (uint64_t c = 0; c < nlist; ++c) {
                double s2 = 0.0;
                for (uint64_t j = 0; j < D; ++j)
                    s2 += (double)h_centroids[c * D + j] * (double)h_centroids[c * D + j];
                cn[c] = static_cast<float>(s2);
                mx = std::max(mx, std::sqrt(s2));
            }
            cmax = std::nextafter(static_cast<float>(mx), FLT_MAX);
            // zero-padded to a multiple of the probe GEMM's 256-column tile (its epilogue reads
            // whole 32-column chunks as float4)
            cn.resize((nlist + 255) / 256 * 256, 0.0f);
            cnorm2.alloc(cn.size());
            CUDA_TRY(cudaMemcpy(cnorm2.p, cn.data(), cn.size() * 4, cudaMemcpyHostToDevice));
        }
        {
            const std::vector<double> rd(h_rotator, h_rotator + dim * D);  // exact widening
            CUDA_TRY(cudaMemcpy(rotator.p, rd.data(), dim * D * 8, cudaMemcpyHostToDevice));
        }
        cl_start.alloc(nlist);
        cl_size.alloc(nlist);
        CUDA_TRY(cudaMemcpy(cl_start.p, starts.data(), nlist * 4, cudaMemcpyHostToDevice));
        CUDA_TRY(cudaMemcpy(cl_size.p, sizes.data(), nlist * 4, cudaMemcpyHostToDevice));
        this->h_ids.assign(h_ids, h_ids + N);
        // The adapter's arrays are staged through bounded buffers, a batch of whole clusters
        // (at most kLoadBatch vectors, or the largest cluster) at a time, so the device holds
        // the resident index plus one batch during loading: word-major 1-bit codes and
        // float[N][3] factors are repacked into scan planes, the 7-bit ex codes, ex factors
        // and ids into the refine rows and meta words.
        scan4.alloc(N * (G16 + 1));
        rows.alloc(std::max<uint64_t>(N * D / 16, 1));
        meta.alloc(std::max<uint64_t>(N, 1));
        {
            constexpr uint64_t kLoadBatch = 1ull << 23;
            const uint64_t cap_v = std::max<uint64_t>(kLoadBatch, largest);
            const uint64_t W = D / 32;
            DevBuf<uint8_t> tmp_long;
            DevBuf<float2> tmp_exf;
            DevBuf<uint32_t> tmp_ids, tmp_short;
            DevBuf<float> tmp_fac;
            tmp_long.alloc(cap_v * LC);
            tmp_exf.alloc(cap_v);
            tmp_ids.alloc(cap_v);
            tmp_short.alloc(cap_v * W);
            tmp_fac.alloc(cap_v * 3);
            for (uint64_t c0 = 0; c0 < nlist;) {
                const uint64_t v0 = starts[c0];
                uint64_t c1 = c0, v1 = v0;
                while (c1 < nlist && (c1 == c0 || v1 + sizes[c1] - v0 <= cap_v)) v1 += sizes[c1++];
                const uint64_t m = v1 - v0;
                if (m) {
                    CUDA_TRY(cudaMemcpy(tmp_long.p, h_long + v0 * LC, m * LC, cudaMemcpyHostToDevice));
                    CUDA_TRY(cudaMemcpy(tmp_exf.p, h_exf + v0 * 2, m * 8, cudaMemcpyHostToDevice));
                    CUDA_TRY(cudaMemcpy(tmp_ids.p, h_ids + v0, m * 4, cudaMemcpyHostToDevice));
                    CUDA_TRY(cudaMemcpy(tmp_short.p, h_short + v0 * W, m * W * 4,
                                        cudaMemcpyHostToDevice));
                    CUDA_TRY(cudaMemcpy(tmp_fac.p, h_short_factors + v0 * 3, m * 12,
                                        cudaMemcpyHostToDevice));
                    repack_scan_planes(tmp_short.p, tmp_fac.p, c0, c1, v0);
                    build_refine_rows_kernel<<<static_cast<unsigned>(c1 - c0), 256, 0, stream>>>(
                        tmp_long.p, tmp_exf.p, tmp_ids.p, scan4.p, cl_start.p, cl_size.p,
                        static_cast<int>(D), G16, LC, static_cast<uint32_t>(c0), v0,
                        reinterpret_cast<uint8_t *>(rows.p), meta.p);
                    CUDA_TRY(cudaGetLastError());
                    // the staging buffers are reused by the next batch
                    CUDA_TRY(cudaStreamSynchronize(stream));
                }
                c0 = c1;
            }
        }
        {
            std::vector<uint32_t> chunk(nlist + 1, 0);
            for (uint64_t c = 0; c < nlist; ++c) chunk[c + 1] = chunk[c] + (sizes[c] + 31) / 32;
            cl_chunk.alloc(nlist + 1);
            CUDA_TRY(cudaMemcpy(cl_chunk.p, chunk.data(), (nlist + 1) * 4, cudaMemcpyHostToDevice));
            chunk_range.alloc(std::max<uint32_t>(chunk[nlist], 1));
            cl_range.alloc(nlist);
            chunk_ranges_kernel<<<static_cast<unsigned>(nlist), 256, 0, stream>>>(
                scan4.p, cl_start.p, cl_size.p, cl_chunk.p, G16, chunk_range.p, cl_range.p);
            CUDA_TRY(cudaGetLastError());
        }
        CUDA_TRY(cudaStreamSynchronize(stream));
        loaded = true;
        ++ws_gen;
        if (xb_map) build_exact_base();
    }

    // enable_exact_refine (hybrid.cuh:171-178): nullptr turns it off. The reference keeps
    // the host mapping and reads rows during its CPU refinement; here the rows this engine
    // needs are copied into HBM (now, or when the index is loaded), in vector order.
    void enable_exact_refine(const uint8_t *mapping, uint64_t rows, uint64_t bdim,
                             uint64_t stride, uint64_t offset) {
        if (mapping && bdim == dim && rows && stride < bdim * 4)
            fail(CORA_EINVAL, "exact base row stride is shorter than a row");
        if (mapping && metric == 1)
            fail(CORA_EINVAL, "exact refinement is defined for L2 indexes only");
        xb_map = mapping;
        xb_rows = rows;
        xb_dim = bdim;
        xb_stride = stride;
        xb_offset = offset;
        drop_graph();
        ++ws_gen;
        if (!mapping) {
            exact_base.release();
            exact_ok.release();
            return;
        }
        if (loaded) build_exact_base();
    }
    void build_exact_base() {
        const bool same_dim = xb_dim == dim;
        exact_base.alloc(std::max<uint64_t>(N * dim, 1));
        exact_ok.alloc(std::max<uint64_t>(N, 1));
        // rows whose id lies outside the base (or every row when the dimension differs)
        // are marked missing and their candidates dropped, as the reference skips them
        // (cpu_refinement.cpp:169-172)
        const uint64_t chunk = 1 << 16;
        std::vector<float> stage(chunk * dim);
        std::vector<uint8_t> ok(chunk);
        for (uint64_t g0 = 0; g0 < N; g0 += chunk) {
            const uint64_t m = std::min(chunk, N - g0);
            for (uint64_t i = 0; i < m; ++i) {
                const uint64_t pid = h_ids[g0 + i];
                ok[i] = same_dim && pid < xb_rows;
                if (ok[i])
                    std::memcpy(stage.data() + i * dim, xb_map + xb_offset + pid * xb_stride,
                                dim * 4);
                else
                    std::memset(stage.data() + i * dim, 0, dim * 4);
            }
            CUDA_TRY(cudaMemcpy(exact_base.p + g0 * dim, stage.data(), m * dim * 4,
                                cudaMemcpyHostToDevice));
            CUDA_TRY(cudaMemcpy(exact_ok.p + g0, ok.data(), m, cudaMemcpyHostToDevice));
        }
    }

    // Loads the whole index, or (shard_world > 1) only the clusters plan_shards() gives this
    // shard: the others keep their centroids, since every shard probes all of them, but no
    // vectors, and the `owned` mask makes the grouping and vanguard kernels skip them. Each
    // kept cluster's vectors stay in their order, so ties between equal lower bounds break
    // the same way as on an unsharded index.
    void load_any(uint64_t num_vecs, uint64_t d, uint64_t p_d, uint64_t n_centroids,
                  uint64_t ex_b, const float *h_centroids, const float *h_rotator,
                  const uint32_t *h_short, const float *h_sf, const uint8_t *h_long,
                  const float *h_exf, const uint32_t *h_ids, const uint64_t *h_sizes) {
        const bool valid = h_centroids && h_rotator && h_short && h_sf && h_long && h_exf &&
                           h_ids && h_sizes && n_centroids && ex_b == 7 && p_d >= d && d &&
                           p_d % 64 == 0 && p_d <= kMaxPaddedDim;
        if (shard_world <= 1 || !valid) {  // invalid arguments: load() reports them
            load(num_vecs, d, p_d, n_centroids, ex_b, h_centroids, h_rotator, h_short, h_sf,
                 h_long, h_exf, h_ids, h_sizes);
            shard_clusters = n_centroids;
            return;
        }
        if (loaded) fail(CORA_ESTATE, "index already loaded");
        uint64_t total = 0;
        for (uint64_t c = 0; c < n_centroids; ++c) {
            if (h_sizes[c] > num_vecs - total) fail(CORA_EINVAL, "cluster sizes exceed index size");
            total += h_sizes[c];
        }
        if (total != num_vecs) fail(CORA_EINVAL, "cluster sizes differ from index size");
        std::vector<int32_t> owner(n_centroids);
        plan_shards(h_sizes, n_centroids, shard_world, owner.data());
        const uint64_t W = p_d / 32, lc = p_d * ex_b / 8;
        uint64_t local = 0, kept = 0;
        for (uint64_t c = 0; c < n_centroids; ++c)
            if (owner[c] == static_cast<int32_t>(shard_rank)) {
                local += h_sizes[c];
                ++kept;
            }
        std::vector<uint32_t> s_short(local * W), s_ids(local);
        std::vector<float> s_sf(local * 3), s_exf(local * 2);
        std::vector<uint8_t> s_long(local * lc), mask(n_centroids, 0);
        std::vector<uint64_t> s_sizes(n_centroids, 0);
        uint64_t src = 0, dst = 0;
        for (uint64_t c = 0; c < n_centroids; ++c) {
            const uint64_t n = h_sizes[c];
            if (owner[c] == static_cast<int32_t>(shard_rank)) {
                // a cluster's 1-bit block is contiguous (word-major within the cluster)
                std::memcpy(s_short.data() + dst * W, h_short + src * W, n * W * 4);
                std::memcpy(s_sf.data() + dst * 3, h_sf + src * 3, n * 12);
                std::memcpy(s_long.data() + dst * lc, h_long + src * lc, n * lc);
                std::memcpy(s_exf.data() + dst * 2, h_exf + src * 2, n * 8);
                std::memcpy(s_ids.data() + dst, h_ids + src, n * 4);
                s_sizes[c] = n;
                mask[c] = 1;
                dst += n;
            }
            src += n;
        }
        load_shard_local(local, d, p_d, n_centroids, ex_b, h_centroids, h_rotator, s_short.data(),
                         s_sf.data(), s_long.data(), s_exf.data(), s_ids.data(), s_sizes.data(),
                         mask, kept);
    }

    // A shard's part of an index, already sliced (sizes 0 outside the shard, `mask` 1 on its
    // clusters): loaded like a whole index, plus the ownership mask.
    void load_shard_local(uint64_t local, uint64_t d, uint64_t p_d, uint64_t n_centroids,
                          uint64_t ex_b, const float *h_centroids, const float *h_rotator,
                          const uint32_t *h_short, const float *h_sf, const uint8_t *h_long,
                          const float *h_exf, const uint32_t *h_ids, const uint64_t *h_sizes,
                          const std::vector<uint8_t> &mask, uint64_t kept) {
        if (local == 0)
            fail(CORA_EINVAL, "shard " + std::to_string(shard_rank) + " of " +
                                  std::to_string(shard_world) +
                                  " owns no vectors; use fewer shards for this index");
        load(local, d, p_d, n_centroids, ex_b, h_centroids, h_rotator, h_short, h_sf, h_long,
             h_exf, h_ids, h_sizes);
        owned.alloc(n_centroids);
        CUDA_TRY(cudaMemcpy(owned.p, mask.data(), n_centroids, cudaMemcpyHostToDevice));
        shard_clusters = kept;
    }

    // Scan planes of clusters [c0, c1) from a staged batch whose first vector is v0.
    void repack_scan_planes(const uint32_t *d_short, const float *d_fac, uint64_t c0, uint64_t c1,
                            uint64_t v0);

    // ---------------------------------------------------------------- workspace
    uint64_t vanguard_depth(uint64_t nprobe) const {
        const uint64_t v = std::max<uint64_t>(vanguard, 1);
        return std::min(v, nprobe);
    }

    void prepare_workspace(uint64_t max_q, uint64_t max_k, uint64_t max_np) {
        if (!loaded) fail(CORA_ESTATE, "load an index before preparing workspace");
        validate_search_shape(max_q, max_k, max_np, nlist, D);
        if (max_k > kMaxTopk) fail(CORA_EINVAL, "topk above 4096 is not supported");
        if (max_np > kMaxProbeFast) fail(CORA_EINVAL, "nprobe above 4096 is not supported");
        free_workspace();
        CUDA_TRY(cudaSetDevice(device));
        ws_q = max_q;
        ws_k = max_k;
        ws_np = max_np;
        ws_vg = vanguard_depth(max_np);
        const uint64_t pool = queue_capacity + spill_capacity;
        const uint64_t keep = std::max<uint64_t>(max_k, kVanguardMinKeep);
        cap = std::max<uint64_t>(1, pool / max_q);
        cap = std::min<uint64_t>(cap, max_np * max_cluster + ws_vg * keep);
        cap = std::min<uint64_t>(cap, UINT32_MAX / 2);
        raw_q.alloc(max_q * dim);
        qr.alloc(max_q * D);
        scal.alloc(max_q);
        ipm.alloc(max_q);
        lut.alloc(max_q * 4 * D);
        planes.alloc(max_q * 8 * W4);
        gmat.alloc(max_q * approx_ld(nlist));
        cmin.alloc(max_q * chunk_stride(static_cast<int>(nlist)));
        qnorm2.alloc(max_q);
        probe_ids.alloc(max_q * max_np);
        probe_g.alloc(max_q * max_np);
        probe_ga.alloc(max_q * max_np);
        T0.alloc(max_q);
        T1.alloc(max_q);
        Tcap.alloc(max_q);
        bound.alloc(max_q * std::max<uint64_t>(ws_vg, 1));
        vg_off.alloc(max_q * std::max<uint64_t>(ws_vg, 1) + 1);
        select_fallback.alloc(max_q * std::max<uint64_t>(ws_vg, 1) + 1);
        filt_list.alloc(max_q * std::max<uint64_t>(ws_vg, 1) + 1);
        {
            // worst case of the lows buffer: every query probes the ws_vg largest clusters
            uint64_t worst = 0;
            for (uint64_t r = 0; r < ws_vg && r < h_sizes_sorted.size(); ++r)
                worst += lows_slice(h_sizes_sorted[r]);  // slices padded to 4 floats
            worst *= max_q;
            size_t free_b = 0, total_b = 0;
            CUDA_TRY(cudaMemGetInfo(&free_b, &total_b));
            const uint64_t limit = std::min<uint64_t>(lows_budget, free_b / 4);
            if (worst > 0 && worst * 4 <= limit) lows.alloc(worst);
        }
        lows_top.alloc(1);
        cand_cnt.alloc(max_q);
        seed_cnt.alloc(max_q);
        cand_rec.alloc(max_q * cap);
        cand_key.alloc(max_q * cap);
        pair_cnt.alloc(nlist);
        pair_off.alloc(nlist + 1);
        pair_cur.alloc(nlist);
        item_off.alloc(nlist);
        pairs.alloc(max_q * max_np);
        items.alloc(max_q * max_np);  // at most one item per pair
        n_items.alloc(1);
        item_counter.alloc(1);
        err.alloc(1);
        stats.alloc(2);
        out_d.alloc(max_q * max_k);
        out_i.alloc(max_q * max_k);
        h_T0.assign(max_q, FLT_MAX);
        CUDA_TRY(cudaMemcpy(T0.p, h_T0.data(), max_q * 4, cudaMemcpyHostToDevice));
        ws_ready = true;
    }

    void free_workspace() noexcept {
        drop_graph();
        ++ws_gen;
        ws_ready = false;
        ws_q = ws_k = ws_np = ws_vg = cap = 0;
        for (auto *b : {&raw_q, &qr, &qnorm2, &gmat, &cmin, &probe_g, &probe_ga, &T0, &T1, &Tcap,
                        &out_d})
            b->release();
        scal.release();
        ipm.release();
        lut.release();
        for (auto *b : {&planes, &cand_cnt, &seed_cnt, &pair_cnt, &pair_off, &pair_cur, &item_off,
                        &pairs, &n_items, &out_i})
            b->release();
        probe_ids.release();
        item_counter.release();
        err.release();
        bound.release();
        vg_off.release();
        lows_top.release();
        select_fallback.release();
        filt_list.release();
        lows.release();
        cand_rec.release();
        cand_key.release();
        items.release();
        stats.release();
        h_T0.clear();
    }

    void require_ws() const {
        if (!ws_ready) fail(CORA_ESTATE, "prepare workspace before searching");
    }
    void validate_ws(uint64_t q, uint64_t k, uint64_t np) const {
        require_ws();
        if (q == 0 || q > ws_q || k == 0 || k > ws_k || np == 0 || np > ws_np)
            fail(CORA_EINVAL, "search shape exceeds the prepared workspace");
    }

    void set_vanguard(uint64_t size) {
        if (ws_ready && vanguard_depth_for(size, ws_np) > ws_vg)
            fail(CORA_ESTATE, "prepare workspace again before increasing vanguard size");
        vanguard = size;
    }
    static uint64_t vanguard_depth_for(uint64_t v, uint64_t np) {
        return std::min<uint64_t>(std::max<uint64_t>(v, 1), np);
    }

    void reset_buffer(const float *h_q, uint64_t nq) {
        validate_ws(nq, 1, 1);
        if (!h_q) fail(CORA_EINVAL, "missing queries");
        CUDA_TRY(cudaSetDevice(device));
        CUDA_TRY(cudaMemcpyAsync(raw_q.p, h_q, nq * dim * 4, cudaMemcpyHostToDevice, stream));
        std::fill(h_T0.begin(), h_T0.end(), FLT_MAX);
        CUDA_TRY(cudaMemcpyAsync(T0.p, h_T0.data(), ws_q * 4, cudaMemcpyHostToDevice, stream));
        CUDA_TRY(cudaMemcpyAsync(Tcap.p, h_T0.data(), ws_q * 4, cudaMemcpyHostToDevice, stream));
        CUDA_TRY(cudaStreamSynchronize(stream));
    }
    void seed_thresholds(const float *in, uint64_t nq) {
        validate_ws(nq, 1, 1);
        if (!in) fail(CORA_EINVAL, "missing threshold input");
        CUDA_TRY(cudaSetDevice(device));
        std::copy(in, in + nq, h_T0.begin());
        CUDA_TRY(cudaMemcpyAsync(T0.p, in, nq * 4, cudaMemcpyHostToDevice, stream));
        CUDA_TRY(cudaMemcpyAsync(Tcap.p, in, nq * 4, cudaMemcpyHostToDevice, stream));
        CUDA_TRY(cudaStreamSynchronize(stream));
    }
    void capture_thresholds(float *out, uint64_t nq) const {
        validate_ws(nq, 1, 1);
        if (!out) fail(CORA_EINVAL, "missing threshold output");
        CUDA_TRY(cudaMemcpy(out, Tcap.p, nq * 4, cudaMemcpyDeviceToHost));
    }

    // ---------------------------------------------------------------- search
    void enqueue_search(const float *d_q, uint64_t nq, uint64_t k, uint64_t np, float *d_od,
                        uint32_t *d_oi, cudaStream_t st);
    void enqueue_front(const float *d_q, uint64_t nq, uint64_t k, uint64_t np, cudaStream_t st,
                       uint64_t *seed_keys_out);
    void enqueue_rotate(const float *d_q, uint64_t nq, uint64_t k, uint64_t np, cudaStream_t st);
    void enqueue_probe_range(uint64_t q0, uint64_t q1, cudaStream_t st);
    void enqueue_probe_gadd(cudaStream_t st);
    void enqueue_vanguard(uint64_t *seed_keys_out);
    void enqueue_back(const uint64_t *seed_recv, int world, float *d_od, uint32_t *d_oi,
                      uint64_t *topk_keys_out);
    void enqueue_final(const uint64_t *topk_recv, int world, float *d_od, uint32_t *d_oi);
    void launch_topk(int mode, float *d_od, uint32_t *d_oi, uint64_t *keys_out, cudaStream_t st);
    IndexView index_view() const;
    SearchView search_view() const;
    ScanLaunch scan_launch(const IndexView &ix, const SearchView &sv, cudaStream_t st) const;
    void group_pairs(int r_lo, int r_hi, bool prune, cudaStream_t st);
    // u64 words per shard in an exchange buffer: k keys per query + one status word.
    static uint64_t exchange_stride(uint64_t nq, uint64_t k) { return nq * k + 1; }
    void finish(cudaStream_t st) {
        int h_err = 0;
        unsigned long long h_stats[2] = {0, 0};
        CUDA_TRY(cudaMemcpyAsync(&h_err, err.p, 4, cudaMemcpyDeviceToHost, st));
        CUDA_TRY(cudaMemcpyAsync(h_stats, stats.p, 16, cudaMemcpyDeviceToHost, st));
        CUDA_TRY(cudaStreamSynchronize(st));
        last_submitted = h_stats[0];
        last_refined = h_stats[0];
        if (gpu_filter_timing) CUDA_TRY(cudaEventElapsedTime(&last_filter_ms, ev_filter0, ev_filter1));
        if (h_err & kDevCandidateOverflow)
            fail(CORA_ERUNTIME,
                 "HBM queue spill capacity exhausted; increase --queue-capacity or "
                 "--queue-spill-capacity, or reduce --query-chunk.");
        if (h_err & kDevWaitTimeout) fail(CORA_ERUNTIME, "a device-side wait timed out");
        if (h_err) fail(CORA_ERUNTIME, "device reported an error");
    }

    void set_metric(int m) {
        if (m != 0 && m != 1) fail(CORA_EINVAL, "metric must be 0 (L2) or 1 (inner product)");
        if (m == 1 && xb_map)
            fail(CORA_EINVAL, "exact refinement is defined for L2 indexes only");
        metric = m;
    }

    void require_whole_index() const {
        if (shard_world > 1)
            fail(CORA_ESTATE, "this engine holds one shard of the index: search it with the "
                              "shard search calls (begin / resume / end) on every shard");
    }

    void search_host(const float *h_q, uint64_t nq, uint64_t k, uint64_t np, float *h_d,
                     uint32_t *h_i, int batch_q) {
        validate_ws(nq, k, np);
        require_whole_index();
        if (!h_q || !h_d || !h_i || batch_q < 1 || batch_q > 6)
            fail(CORA_EINVAL, "invalid search buffers or batch-q (expected 1..6)");
        CUDA_TRY(cudaSetDevice(device));
        CUDA_TRY(cudaMemcpyAsync(raw_q.p, h_q, nq * dim * 4, cudaMemcpyHostToDevice, stream));
        enqueue_search(raw_q.p, nq, k, np, out_d.p, out_i.p, stream);
        CUDA_TRY(cudaMemcpyAsync(h_d, out_d.p, nq * k * 4, cudaMemcpyDeviceToHost, stream));
        CUDA_TRY(cudaMemcpyAsync(h_i, out_i.p, nq * k * 4, cudaMemcpyDeviceToHost, stream));
        finish(stream);
    }

    void debug_copy(int what, void *out, uint64_t bytes);

    // Stage boundary events, recorded only when profiling is enabled.
    void accumulate_set(int set) {
        float ms;
        for (int i = 0; i < kStages; ++i) {
            CUDA_TRY(cudaEventSynchronize(ev_stage[set][i + 1]));
            CUDA_TRY(cudaEventElapsedTime(&ms, ev_stage[set][i], ev_stage[set][i + 1]));
            stage_sum[i] += ms;
        }
        ++stage_count;
    }
    void begin_profiled_search() {
        if (!profiling) return;
        if (ring_used == kRing) accumulate_set(ring_next);  // recorded kRing searches ago
        else ++ring_used;
        ring_last = ring_next;
        ring_next = (ring_next + 1) % kRing;
    }
    void mark(int i, cudaStream_t st) {
        if (profiling) CUDA_TRY(cudaEventRecord(ev_stage[ring_last][i], st));
    }
    void stage_ms(float *out, uint64_t n) {
        if (ring_last < 0) fail(CORA_ESTATE, "no profiled search recorded");
        if (n > kStages) n = kStages;
        CUDA_TRY(cudaEventSynchronize(ev_stage[ring_last][kStages]));
        for (uint64_t i = 0; i < n; ++i)
            CUDA_TRY(cudaEventElapsedTime(out + i, ev_stage[ring_last][i], ev_stage[ring_last][i + 1]));
    }
    // Sums of every profiled search since the last reset (flushes the ring).
    uint64_t stage_totals(double *out, uint64_t n) {
        while (ring_used > 0) {
            const int set = (ring_next - ring_used + kRing) % kRing;
            accumulate_set(set);
            --ring_used;
        }
        if (n > kStages) n = kStages;
        for (uint64_t i = 0; i < n; ++i) out[i] = stage_sum[i];
        return stage_count;
    }
    void stage_reset() {
        ring_used = 0;
        ring_last = -1;
        stage_count = 0;
        for (auto &v : stage_sum) v = 0.0;
    }
};

// ------------------------------------------------------------------------------------
// repack: adapter layout -> scan planes (one CTA per cluster)
// ------------------------------------------------------------------------------------
// short_data / fac hold a staged batch of whole clusters starting at vector v0; this launch
// covers clusters c0 + blockIdx.x.
__global__ void repack_kernel(const uint32_t *__restrict__ short_data,
                              const float *__restrict__ fac, const uint32_t *__restrict__ cl_start,
                              const uint32_t *__restrict__ cl_size, int W, int G16, uint32_t c0,
                              uint64_t v0, uint4 *__restrict__ scan4) {
    const uint32_t c = c0 + blockIdx.x;
    const uint32_t s = cl_start[c], n = cl_size[c];
    const uint64_t ls = s - v0;  // the cluster's first vector within the batch
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        for (int g = 0; g < G16; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int word = 4 * g + t;
                w[t] = word < W ? short_data[ls * W + (size_t)word * n + i] : 0u;
            }
            scan4[(size_t)(G16 + 1) * s + (size_t)g * n + i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
        const float *f = fac + (ls + i) * 3;
        scan4[(size_t)(G16 + 1) * s + (size_t)G16 * n + i] =
            make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]), 0u);
    }
}

void Engine::repack_scan_planes(const uint32_t *d_short, const float *d_fac, uint64_t c0,
                                uint64_t c1, uint64_t v0) {
    repack_kernel<<<static_cast<unsigned>(c1 - c0), 256, 0, stream>>>(
        d_short, d_fac, cl_start.p, cl_size.p, static_cast<int>(D / 32), G16,
        static_cast<uint32_t>(c0), v0, scan4.p);
    CUDA_TRY(cudaGetLastError());
}

// ------------------------------------------------------------------------------------
// search pipeline
// ------------------------------------------------------------------------------------
namespace {
// Query words per pair in the scan kernels' shared memory (bytes): integer estimator 8 W4
// words, LUT estimator kLutFloats table entries.
template <int G16, bool kLut>
constexpr size_t query_block_bytes() {
    return kLut ? (size_t)ScanShape<G16>::kLutFloats * 4 : (size_t)8 * ScanShape<G16>::W4 * 4;
}
template <int G16, bool kLut>
size_t rescan_smem(int sort_n) {
    using Sh = ScanShape<G16>;
    return 2 * Sh::kStageEntries * 16 + query_block_bytes<G16, kLut>() + (size_t)sort_n * 8;
}
template <int G16, bool kLut>
size_t scan_smem() {
    using Sh = ScanShape<G16>;
    const int ppi = kLut ? Sh::kLutPairs : kMaxPairsPerItem;
    return (size_t)Sh::kStages * Sh::kScanStageEntries * 16 +
           (size_t)ppi * query_block_bytes<G16, kLut>();
}

template <int G16, bool kLows, bool kLut>
void launch_grouped(const ScanLaunch &L) {
    const size_t sm = scan_smem<G16, kLut>();
    auto *kern = scan_kernel<G16, kLows, kLut>;
    CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    int per_sm = 0;
    CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kScanThreads, sm));
    const int grid = std::max(1, per_sm) * L.num_sms;
    kern<<<grid, kScanThreads, sm, L.st>>>(L.ix, L.sv, L.items, L.n_items, L.pairs,
                                           L.item_counter);
    CUDA_TRY(cudaGetLastError());
}

template <int G16, bool kLut>
void launch_scan(const ScanLaunch &L, ScanPhase phase) {
    if (phase == ScanPhase::kRescanVanguard) {
        const size_t sm = rescan_smem<G16, kLut>(L.rescan_sort_n);
        auto *kern = vanguard_rescan_kernel<G16, kLut>;
        CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        kern<<<static_cast<unsigned>(L.n_van), kScanThreads, sm, L.st>>>(L.ix, L.sv,
                                                                         L.rescan_sort_n, L.owned);
        CUDA_TRY(cudaGetLastError());
    } else if (phase == ScanPhase::kWriteLows) {
        launch_grouped<G16, true, kLut>(L);
    } else {
        launch_grouped<G16, false, kLut>(L);
    }
}

void dispatch_scan(int G16, bool lut, const ScanLaunch &L, ScanPhase phase) {
#define CORA_SCAN_CASE(G)                    \
    case G:                                  \
        if (lut)                             \
            launch_scan<G, true>(L, phase);  \
        else                                 \
            launch_scan<G, false>(L, phase); \
        break;
    switch (G16) {
        CORA_SCAN_CASE(1)
        CORA_SCAN_CASE(2)
        CORA_SCAN_CASE(3)
        CORA_SCAN_CASE(4)
        CORA_SCAN_CASE(5)
        CORA_SCAN_CASE(6)
        CORA_SCAN_CASE(7)
        CORA_SCAN_CASE(8)
        default: fail(CORA_EINVAL, "unsupported padded dimension");
    }
#undef CORA_SCAN_CASE
}

// Pairs per grouped item with the LUT estimator (ScanShape::kLutPairs).
int lut_pairs_per_item(int G16) { return G16 == 1 ? 32 : (G16 == 2 ? 16 : 8); }
}  // namespace

IndexView Engine::index_view() const {
    return IndexView{scan4.p, cl_start.p, cl_size.p, chunk_range.p, cl_chunk.p, cl_range.p,
                     rows.p, meta.p, exact_base.n ? exact_base.p : nullptr, exact_ok.p,
                     static_cast<int>(nlist), static_cast<int>(D), G16, LC, static_cast<int>(dim)};
}

SearchView Engine::search_view() const {
    const uint64_t veff = vanguard_depth(last_np);
    const uint64_t keep = std::max<uint64_t>(last_k, kVanguardMinKeep);
    return SearchView{static_cast<int>(last_nq), static_cast<int>(last_k), static_cast<int>(last_np),
                      static_cast<int>(veff), static_cast<int>(keep), static_cast<int>(cap),
                      last_dq, scal.p, ipm.p, planes.p, lut.p, lut_mode() ? 1 : 0, qr.p,
                      probe_ids.p, probe_g.p, metric == 1 ? probe_ga.p : probe_g.p, T0.p, Tcap.p,
                      T1.p, bound.p,
                      cand_cnt.p, seed_cnt.p, cand_rec.p, cand_key.p, lows.p, vg_off.p, lows.n,
                      lows_top.p, err.p, warp_select_limit, topk_warp_limit,
                      refine_full_code ? 1 : 0};
}

void Engine::enqueue_search(const float *d_q, uint64_t nq, uint64_t k, uint64_t np, float *d_od,
                            uint32_t *d_oi, cudaStream_t st) {
    // graphs need a capturable stream, and stage events / filter timing stay eager
    const bool special = st == nullptr || st == cudaStreamLegacy || st == cudaStreamPerThread;
    if (!search_graphs || profiling || gpu_filter_timing || special) {
        enqueue_front(d_q, nq, k, np, st, nullptr);
        enqueue_back(nullptr, 0, d_od, d_oi, nullptr);
        mark(13, st);
        return;
    }
    GraphKey key;
    key.d_q = d_q;
    key.nq = nq;
    key.k = k;
    key.np = np;
    key.ws_gen = ws_gen;
    key.vanguard = vanguard;
    key.d_od = d_od;
    key.d_oi = d_oi;
    key.st = st;
    key.wsl = warp_select_limit;
    key.twl = topk_warp_limit;
    key.rl = refine_lanes;
    key.reuse = cross_query_reuse;
    key.full_code = refine_full_code;
    key.lut = lut_mode();
    key.metric = metric;
    if (!graph_exec || !graph_key.same(key)) {
        drop_graph();
        CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
        try {
            enqueue_front(d_q, nq, k, np, st, nullptr);
            enqueue_back(nullptr, 0, d_od, d_oi, nullptr);
        } catch (...) {
            cudaGraph_t broken = nullptr;
            cudaStreamEndCapture(st, &broken);
            if (broken) cudaGraphDestroy(broken);
            throw;
        }
        cudaGraph_t g = nullptr;
        CUDA_TRY(cudaStreamEndCapture(st, &g));
        const cudaError_t ie = cudaGraphInstantiate(&graph_exec, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
            graph_exec = nullptr;
            CUDA_TRY(ie);
        }
        graph_key = key;
    }
    // the host-side record of the search that the eager path keeps
    last_stream = st;
    last_nq = nq;
    last_k = k;
    last_np = np;
    last_dq = d_q;
    CUDA_TRY(cudaGraphLaunch(graph_exec, st));
}

// Stages 0..7: rotation, probing, vanguard seeding and seed refinement, then the threshold
// (T1) or, for a sharded search, this shard's k smallest seed keys into seed_keys_out.
void Engine::enqueue_front(const float *d_q, uint64_t nq, uint64_t k, uint64_t np,
                           cudaStream_t st, uint64_t *seed_keys_out) {
    enqueue_rotate(d_q, nq, k, np, st);
    enqueue_probe_range(0, nq, st);
    enqueue_probe_gadd(st);
    mark(3, st);
    enqueue_vanguard(seed_keys_out);
}

// Steps 0-1 of a search: counters, rotation, query factors, bit-planes (and LUT tables) of
// every query of the batch.
void Engine::enqueue_rotate(const float *d_q, uint64_t nq, uint64_t k, uint64_t np,
                            cudaStream_t st) {
    last_stream = st;
    last_nq = nq;
    last_k = k;
    last_np = np;
    last_dq = d_q;
    CUDA_TRY(cudaMemsetAsync(err.p, 0, 4, st));
    CUDA_TRY(cudaMemsetAsync(stats.p, 0, 16, st));
    CUDA_TRY(cudaMemsetAsync(cand_cnt.p, 0, nq * 4, st));
    begin_profiled_search();
    mark(0, st);

    // 1. rotation + query factors + bit-planes
    {
        const float c_b = -static_cast<float>((1u << (ex_bits + 1)) - 1u) / 2.0f;
        launch_rotate_prep(d_q, nq, dim, D, W4, rotator.p, c_b, qr.p, scal.p, planes.p, qnorm2.p,
                           ipm.p, st);
        if (lut_mode()) {  // the LUT estimator's tables (and its pruning bound, over ipm)
            lut_build_kernel<<<static_cast<unsigned>((nq + kLutWarps - 1) / kLutWarps),
                               32 * kLutWarps, 0, st>>>(qr.p, scal.p, static_cast<int>(nq),
                                                        static_cast<int>(D), lut.p, ipm.p);
            CUDA_TRY(cudaGetLastError());
        }
    }
    mark(1, st);
}

// Step 2 for queries [q0, q1) of the batch: approximate distances for every (query,
// centroid) on the tensor cores, then the exact top-nprobe among the guarded candidates.
void Engine::enqueue_probe_range(uint64_t q0, uint64_t q1, cudaStream_t st) {
    const uint64_t np = last_np, m = q1 - q0;
    if (m > 0) {
        launch_probe_gemm(qr.p + q0 * D, qnorm2.p + q0, m, D, centroids.p, cnorm2.p, nlist,
                          gmat.p, cmin.p, num_sms, st, err.p);
        mark(2, st);
        // select_fallback (>= 1 + nq words) is free until the vanguard stage
        launch_guarded_select(gmat.p, cmin.p, nlist, m, np, qr.p + q0 * D, qnorm2.p + q0,
                              centroids.p, cmax, D, probe_ids.p + q0 * np, probe_g.p + q0 * np,
                              select_fallback.p, num_sms, st);
    } else {
        mark(2, st);
    }
}

// Inner product: the additive term -<q', c'> of every probe of the batch.
void Engine::enqueue_probe_gadd(cudaStream_t st) {
    if (metric != 1) return;
    const uint64_t nq = last_nq;
    ip_gadd_kernel<<<static_cast<unsigned>((nq + 7) / 8), 256, 0, st>>>(
        qr.p, centroids.p, probe_ids.p, static_cast<int>(nq), static_cast<int>(last_np),
        static_cast<int>(D), probe_ga.p);
    CUDA_TRY(cudaGetLastError());
}

// Steps 3-5 of a search (probe lists in place): the vanguard pairs' seeds, their refinement
// and the threshold (or, sharded, this shard's k smallest seed keys into seed_keys_out).
void Engine::enqueue_vanguard(uint64_t *seed_keys_out) {
    cudaStream_t st = last_stream;
    const uint64_t nq = last_nq, k = last_k, np = last_np;
    const int inq = static_cast<int>(nq);
    const uint64_t veff = vanguard_depth(np);
    const uint64_t keep = std::max<uint64_t>(k, kVanguardMinKeep);
    const bool lows_mode = lows.n > 0;
    const IndexView ix = index_view();
    const SearchView sv = search_view();
    const uint8_t *own = owned.n ? owned.p : nullptr;
    const ScanLaunch L = scan_launch(ix, sv, st);
    const int iveff = static_cast<int>(veff);
    const unsigned n_van = static_cast<unsigned>(nq * veff);
    // 3. vanguard pairs: seeds (best `keep` keys per pair among low < T0)
    if (lows_mode) {
        group_pairs(0, iveff, false, st);
        // the lows pass bump-allocates the pairs' slices
        CUDA_TRY(cudaMemsetAsync(lows_top.p, 0, sizeof(unsigned long long), st));
    }
    mark(4, st);
    if (gpu_filter_timing) CUDA_TRY(cudaEventRecord(ev_filter0, st));
    if (lows_mode)
        dispatch_scan(G16, lut_mode(), L, ScanPhase::kWriteLows);
    else
        dispatch_scan(G16, lut_mode(), L, ScanPhase::kRescanVanguard);
    mark(5, st);
    if (lows_mode) {
        const size_t sm = (size_t)next_pow2(static_cast<int>(keep)) * 8 + kSelectStage * 4;
        CUDA_TRY(cudaFuncSetAttribute(vanguard_select_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        if (keep <= static_cast<uint64_t>(kWarpSelectMax)) {
            // one warp per pair; the rare pair with too many keys below the first bound
            // is finished by a grid-stride block selection over the queued list
            CUDA_TRY(cudaMemsetAsync(select_fallback.p, 0, 4, st));
            const unsigned grid = (n_van + 7) / 8;
            if (keep <= 32)
                vanguard_select_warp_kernel<1><<<grid, 256, 0, st>>>(ix, sv, own, select_fallback.p);
            else if (keep <= 64)
                vanguard_select_warp_kernel<2><<<grid, 256, 0, st>>>(ix, sv, own, select_fallback.p);
            else
                vanguard_select_warp_kernel<4><<<grid, 256, 0, st>>>(ix, sv, own, select_fallback.p);
            CUDA_TRY(cudaGetLastError());
            vanguard_select_kernel<<<static_cast<unsigned>(2 * num_sms), 256, sm, st>>>(
                ix, sv, own, select_fallback.p);
        } else {
            vanguard_select_kernel<<<n_van, 256, sm, st>>>(ix, sv, own, nullptr);
        }
        CUDA_TRY(cudaGetLastError());
    }
    mark(6, st);
    launch_refine(ix, sv, static_cast<int>(D), static_cast<int>(np), 0, inq, refine_lanes, st);
    CUDA_TRY(cudaGetLastError());
    mark(7, st);
    launch_topk(0, nullptr, nullptr, seed_keys_out, st);
}

// Threshold (mode 0) or final top-k (mode 1): one warp per query for k <= 32 (the queries
// whose candidate collection overflows go on to the block kernel through select_fallback,
// free at this point), else one CTA per query.
void Engine::launch_topk(int mode, float *d_od, uint32_t *d_oi, uint64_t *keys_out,
                         cudaStream_t st) {
    const SearchView sv = search_view();
    const unsigned inq = static_cast<unsigned>(last_nq);
    const size_t sel_sm = (size_t)next_pow2(static_cast<int>(last_k)) * 8;
    CUDA_TRY(cudaFuncSetAttribute(threshold_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sel_sm));
    CUDA_TRY(cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)sel_sm));
    if (last_k <= 32) {
        CUDA_TRY(cudaMemsetAsync(select_fallback.p, 0, 4, st));
        topk_warp_kernel<<<(inq + 7) / 8, 256, 0, st>>>(sv, mode, d_od, d_oi, stats.p, keys_out,
                                                          select_fallback.p);
        CUDA_TRY(cudaGetLastError());
        const unsigned grid = static_cast<unsigned>(2 * num_sms);
        if (mode == 0)
            threshold_kernel<<<grid, 256, sel_sm, st>>>(sv, keys_out, select_fallback.p);
        else
            merge_kernel<<<grid, 256, sel_sm, st>>>(sv, d_od, d_oi, nullptr, keys_out,
                                                     select_fallback.p);
    } else if (mode == 0) {
        threshold_kernel<<<inq, 256, sel_sm, st>>>(sv, keys_out, nullptr);
    } else {
        merge_kernel<<<inq, 256, sel_sm, st>>>(sv, d_od, d_oi, stats.p, keys_out, nullptr);
    }
    CUDA_TRY(cudaGetLastError());
}

ScanLaunch Engine::scan_launch(const IndexView &ix, const SearchView &sv, cudaStream_t st) const {
    const uint64_t keep = std::max<uint64_t>(last_k, kVanguardMinKeep);
    const int rescan_sort_n = next_pow2(static_cast<int>(keep) + 256 /* ScanShape::TV */);
    return ScanLaunch{ix, sv, rescan_sort_n, last_nq * vanguard_depth(last_np), items.p, n_items.p,
                      pairs.p, item_counter.p, owned.n ? owned.p : nullptr, num_sms, st};
}

// Per-cluster grouping of the (query, probe rank) pairs with rank in [r_lo, r_hi): cross-query
// reuse serves up to kMaxPairsPerItem queries from one cluster read.
// prune: leave out the pairs that pair_pruned proves candidate-free against T1 (main pass).
void Engine::group_pairs(int r_lo, int r_hi, bool prune, cudaStream_t st) {
    const int inq = static_cast<int>(last_nq), inp = static_cast<int>(last_np);
    const uint8_t *own = owned.n ? owned.p : nullptr;
    const size_t total = last_nq * last_np;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    CUDA_TRY(cudaMemsetAsync(pair_cnt.p, 0, nlist * 4, st));
    CUDA_TRY(cudaMemsetAsync(pair_cur.p, 0, nlist * 4, st));
    CUDA_TRY(cudaMemsetAsync(item_counter.p, 0, 4, st));
    const int ppi = !cross_query_reuse ? 1 : (lut_mode() ? lut_pairs_per_item(G16) : kMaxPairsPerItem);
    PairPrune pp{};
    if (prune)
        pp = PairPrune{cl_range.p, probe_g.p, metric == 1 ? probe_ga.p : probe_g.p, ipm.p, T1.p};
    count_pairs_kernel<<<blocks, 256, 0, st>>>(probe_ids.p, inq, inp, r_lo, r_hi, own, pp,
                                               pair_cnt.p);
    scan_pairs_kernel<<<1, 1024, 0, st>>>(pair_cnt.p, static_cast<int>(nlist), ppi, pair_off.p,
                                           item_off.p, n_items.p);
    scatter_pairs_kernel<<<blocks, 256, 0, st>>>(probe_ids.p, inq, inp, r_lo, r_hi, own, pp,
                                                 pair_off.p, pair_cur.p, pairs.p);
    emit_items_kernel<<<static_cast<unsigned>((nlist + 255) / 256), 256, 0, st>>>(
        pair_cnt.p, pair_off.p, item_off.p, static_cast<int>(nlist), ppi, items.p);
    CUDA_TRY(cudaGetLastError());
}

// Stages 8..12 on last_stream: (sharded: T1 from every shard's seed keys in seed_recv) the
// main pass against T1, refinement and the top-k, written as the result or, sharded, as this
// shard's k best keys (+ its error word) into topk_keys_out.
void Engine::enqueue_back(const uint64_t *seed_recv, int world, float *d_od, uint32_t *d_oi,
                          uint64_t *topk_keys_out) {
    cudaStream_t st = last_stream;
    const int inq = static_cast<int>(last_nq), inp = static_cast<int>(last_np);
    const int iveff = static_cast<int>(vanguard_depth(last_np));
    const unsigned n_van = static_cast<unsigned>(last_nq * vanguard_depth(last_np));
    const bool lows_mode = lows.n > 0;
    const IndexView ix = index_view();
    const SearchView sv = search_view();
    const uint8_t *own = owned.n ? owned.p : nullptr;
    const ScanLaunch L = scan_launch(ix, sv, st);
    const size_t sel_sm = (size_t)next_pow2(static_cast<int>(last_k)) * 8;
    if (seed_recv) {
        CUDA_TRY(cudaFuncSetAttribute(gather_threshold_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sel_sm));
        gather_threshold_kernel<<<inq, 256, sel_sm, st>>>(seed_recv, world,
                                                          exchange_stride(last_nq, last_k), sv);
        CUDA_TRY(cudaGetLastError());
    }
    mark(8, st);
    // 4. main pass against T1: the other probes are scanned; the vanguard probes are either
    //    filtered from their stored lows or rescanned, skipping their seeds in both cases.
    group_pairs(lows_mode ? iveff : 0, inp, true, st);
    mark(9, st);
    dispatch_scan(G16, lut_mode(), L, ScanPhase::kMain);
    mark(10, st);
    if (lows_mode) {
        CUDA_TRY(cudaMemsetAsync(filt_list.p, 0, 4, st));
        filter_list_kernel<<<(n_van + 255) / 256, 256, 0, st>>>(ix, sv, own, filt_list.p);
        vanguard_filter_kernel<<<(n_van + 7) / 8, 256, 0, st>>>(ix, sv, filt_list.p);
        CUDA_TRY(cudaGetLastError());
    }
    if (gpu_filter_timing) CUDA_TRY(cudaEventRecord(ev_filter1, st));
    mark(11, st);
    launch_refine(ix, sv, static_cast<int>(D), static_cast<int>(last_np), 1, inq, refine_lanes, st);
    CUDA_TRY(cudaGetLastError());
    mark(12, st);
    // 5. final top-k
    launch_topk(1, d_od, d_oi, topk_keys_out, st);
}

// Sharded search, last step: the top-k over every shard's k best keys in topk_recv.
void Engine::enqueue_final(const uint64_t *topk_recv, int world, float *d_od, uint32_t *d_oi) {
    cudaStream_t st = last_stream;
    const SearchView sv = search_view();
    const size_t sel_sm = (size_t)next_pow2(static_cast<int>(last_k)) * 8;
    CUDA_TRY(cudaFuncSetAttribute(gather_merge_kernel,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sel_sm));
    gather_merge_kernel<<<static_cast<unsigned>(last_nq), 256, sel_sm, st>>>(
        topk_recv, world, exchange_stride(last_nq, last_k), sv, d_od, d_oi);
    CUDA_TRY(cudaGetLastError());
    mark(13, st);
}

// ------------------------------------------------------------------------------------
// diagnostics
// ------------------------------------------------------------------------------------
void Engine::debug_copy(int what, void *out, uint64_t bytes) {
    require_ws();
    CUDA_TRY(cudaSetDevice(device));
    CUDA_TRY(cudaStreamSynchronize(last_stream));
    const uint64_t nq = last_nq, np = last_np;
    auto copy = [&](const void *src, uint64_t want) {
        if (bytes != want) fail(CORA_EINVAL, "debug_copy: byte count does not match the array");
        CUDA_TRY(cudaMemcpy(out, src, want, cudaMemcpyDeviceToHost));
    };
    switch (what) {
        case 0: copy(qr.p, nq * D * 4); break;
        case 1: copy(probe_ids.p, nq * np * 4); break;
        case 2: copy(probe_g.p, nq * np * 4); break;
        case 3: copy(cand_cnt.p, nq * 4); break;
        case 4: copy(T1.p, nq * 4); break;
        case 5: copy(planes.p, nq * 8 * W4 * 4); break;
        case 6: copy(scal.p, nq * 16); break;
        case 8: copy(gmat.p, nq * approx_ld(nlist) * 4); break;
        case 9: copy(lut.p, nq * 4 * D * 2); break;
        case 10: copy(metric == 1 ? probe_ga.p : probe_g.p, nq * np * 4); break;
        case 7: {
            if (bytes != nq * cap * 4) fail(CORA_EINVAL, "debug_copy: byte count does not match");
            std::vector<uint64_t> rec(nq * cap);
            std::vector<uint32_t> cnt(nq);
            CUDA_TRY(cudaMemcpy(rec.data(), cand_rec.p, nq * cap * 8, cudaMemcpyDeviceToHost));
            CUDA_TRY(cudaMemcpy(cnt.data(), cand_cnt.p, nq * 4, cudaMemcpyDeviceToHost));
            auto *o = static_cast<uint32_t *>(out);
            for (uint64_t q = 0; q < nq; ++q) {
                const uint64_t n = std::min<uint64_t>(cnt[q], cap);
                for (uint64_t i = 0; i < cap; ++i)
                    o[q * cap + i] = i < n ? static_cast<uint32_t>(rec[q * cap + i] & 0xFFFFFFFFu)
                                           : 0xFFFFFFFFu;
                std::sort(o + q * cap, o + q * cap + n);
            }
            break;
        }
        default: fail(CORA_EINVAL, "debug_copy: unknown array");
    }
}

// ------------------------------------------------------------------------------------
// index file -> adapter arrays (ivf.hpp:447-539 + search_data.cpp:45-123)
// ------------------------------------------------------------------------------------
namespace {
// An index file read whole, or (world > 1) only the clusters plan_shards() gives `rank`:
// then num and sizes count this shard's vectors (sizes 0 elsewhere), `owned` marks its
// clusters, and every centroid is kept (each shard probes all of them).
struct FileIndex {
    uint64_t num = 0, dim = 0, nlist = 0, ex_bits = 0, D = 0;
    int metric = 0;  // MetricType byte of the header: 0 L2, 1 IP
    uint64_t full_num = 0, kept = 0, bytes_read = 0;
    std::vector<uint64_t> sizes;
    std::vector<uint8_t> owned;
    std::vector<float> rotator, centroids, short_factors, ex_factors;
    std::vector<uint32_t> short_data, ids;
    std::vector<uint8_t> long_codes;
};

// Centroids of an HNSW-initialised index (nlist >= 20000) from its hnswlib sidecar
// `<index>.hnsw`, written by hnswlib's saveIndex (third_party/.../hnswlib/hnswalg.h:685-713):
// a header of offsetLevel0, max_elements, cur_element_count, size_data_per_element,
// label_offset, offsetData (u64), maxlevel (i32), enterpoint_node (u32), maxM, maxM0, M
// (u64), mult (f64), ef_construction (u64), then cur_element_count level-0 records whose
// vector (D floats) sits at offsetData and label (u64, the cluster id) at label_offset
// (initializer.hpp:207-214). The upper-level links that follow are not needed.
void read_hnsw_centroids(const char *path, uint64_t nlist, uint64_t D, float *out) {
    std::ifstream in(path, std::ios::binary);
    if (!in) fail(CORA_EINVAL, std::string("Cannot open HNSW centroid sidecar: ") + path);
    uint64_t h6[6];
    int32_t maxlevel;
    uint32_t enterpoint;
    uint64_t h3[3];
    double mult;
    uint64_t efc;
    in.read(reinterpret_cast<char *>(h6), sizeof h6);
    in.read(reinterpret_cast<char *>(&maxlevel), 4);
    in.read(reinterpret_cast<char *>(&enterpoint), 4);
    in.read(reinterpret_cast<char *>(h3), sizeof h3);
    in.read(reinterpret_cast<char *>(&mult), 8);
    in.read(reinterpret_cast<char *>(&efc), 8);
    if (!in) fail(CORA_EINVAL, "truncated HNSW centroid sidecar");
    const uint64_t count = h6[2], per = h6[3], label_off = h6[4], data_off = h6[5];
    if (h6[0] != 0 || count != nlist || data_off + 4 * D > per || label_off + 8 > per)
        fail(CORA_EINVAL, "HNSW centroid sidecar does not match the index's clusters");
    std::vector<uint8_t> rec(per);
    std::vector<uint8_t> seen(nlist, 0);
    for (uint64_t i = 0; i < count; ++i) {
        in.read(reinterpret_cast<char *>(rec.data()), static_cast<std::streamsize>(per));
        if (!in) fail(CORA_EINVAL, "truncated HNSW centroid sidecar");
        uint64_t label;
        std::memcpy(&label, rec.data() + label_off, 8);
        if (label >= nlist || seen[label])
            fail(CORA_EINVAL, "HNSW centroid sidecar labels are not the cluster ids");
        seen[label] = 1;
        std::memcpy(out + label * D, rec.data() + data_off, 4 * D);
    }
}

// Reads an IVF index file (ivf.hpp:403-445; centroids embedded, or in the hnswlib sidecar
// for nlist >= 20000). The payload sections (FastScan
// batches, ex codes, ids) are laid out by cluster, so a shard seeks to its own clusters and
// reads each run of consecutive owned clusters in one piece: a shard's host memory and file
// traffic are its share of the index, not the whole file.
FileIndex read_index_file(const char *path, uint32_t rank = 0, uint32_t world = 1) {
    std::ifstream in(path, std::ios::binary);
    if (!in) fail(CORA_EINVAL, std::string("Cannot open IVF index: ") + path);
    FileIndex f;
    uint64_t hdr[4];
    uint8_t types[2];
    in.read(reinterpret_cast<char *>(hdr), sizeof(hdr));
    in.read(reinterpret_cast<char *>(types), 2);
    if (!in) fail(CORA_EINVAL, "truncated IVF index header");
    f.full_num = hdr[0];
    f.dim = hdr[1];
    f.nlist = hdr[2];
    f.ex_bits = hdr[3];
    if (types[0] != 0) fail(CORA_EINVAL, "only matrix-rotator indexes are supported");
    if (types[1] > 1) fail(CORA_EINVAL, "unknown metric type in the IVF index header");
    f.metric = types[1];
    if (!f.full_num || !f.dim || !f.nlist || f.ex_bits > 8)
        fail(CORA_EINVAL, "invalid IVF index header");
    f.D = (f.dim + 63) / 64 * 64;
    const uint64_t D = f.D, W = D / 32;
    std::vector<uint64_t> full_sizes(f.nlist);
    in.read(reinterpret_cast<char *>(full_sizes.data()), 8 * f.nlist);
    uint64_t total = 0, blocks = 0;
    for (auto sz : full_sizes) {
        total += sz;
        blocks += (sz + 31) / 32;
    }
    if (!in || total != f.full_num)
        fail(CORA_EINVAL, "The sum of cluster num != total number of points");
    f.rotator.resize(f.dim * D);
    in.read(reinterpret_cast<char *>(f.rotator.data()), 4 * f.dim * D);
    const std::streampos begin = in.tellg();
    in.seekg(0, std::ios::end);
    const uint64_t remaining = static_cast<uint64_t>(in.tellg() - begin);
    in.seekg(begin);
    const uint64_t rec = D * 4 + 32 * 12;
    const uint64_t ex_stride = f.ex_bits ? D * f.ex_bits / 8 + 8 : 0;
    const uint64_t payload = blocks * rec + f.full_num * ex_stride + 4 * f.full_num;
    const bool sidecar = remaining == payload;  // nlist >= 20000: hnswlib sidecar centroids
    if (!sidecar && remaining != payload + 4 * D * f.nlist)
        fail(CORA_EINVAL, "IVF index size does not match a supported centroid layout");
    f.centroids.resize(f.nlist * D);
    if (sidecar) {
        read_hnsw_centroids((std::string(path) + ".hnsw").c_str(), f.nlist, D, f.centroids.data());
    } else {
        in.read(reinterpret_cast<char *>(f.centroids.data()), 4 * D * f.nlist);
        if (!in) fail(CORA_EINVAL, "Failed to read IVF index payload");
    }
    const uint64_t batch_at = static_cast<uint64_t>(begin) + (sidecar ? 0 : 4 * D * f.nlist);
    const uint64_t ex_at = batch_at + blocks * rec;
    const uint64_t ids_at = ex_at + f.full_num * ex_stride;

    // the clusters this reader keeps, and their local layout
    f.owned.assign(f.nlist, 1);
    if (world > 1) {
        std::vector<int32_t> owner(f.nlist);
        plan_shards(full_sizes.data(), f.nlist, world, owner.data());
        for (uint64_t c = 0; c < f.nlist; ++c) f.owned[c] = owner[c] == static_cast<int32_t>(rank);
    }
    f.sizes.assign(f.nlist, 0);
    std::vector<uint64_t> cstart(f.nlist + 1, 0), bstart(f.nlist + 1, 0), lstart(f.nlist + 1, 0);
    for (uint64_t c = 0; c < f.nlist; ++c) {
        cstart[c + 1] = cstart[c] + full_sizes[c];
        bstart[c + 1] = bstart[c] + (full_sizes[c] + 31) / 32;
        f.sizes[c] = f.owned[c] ? full_sizes[c] : 0;
        lstart[c + 1] = lstart[c] + f.sizes[c];
        f.kept += f.owned[c];
    }
    f.num = lstart[f.nlist];
    const uint64_t lc = D * f.ex_bits / 8;
    f.short_data.assign(f.num * W, 0u);
    f.short_factors.assign(f.num * 3, 0.0f);
    f.long_codes.resize(f.num * lc);
    f.ex_factors.resize(f.num * 2);
    f.ids.resize(f.num);

    // FastScan batches of 32 vectors -> word-major 1-bit codes per cluster. In a batch,
    // dims 8i..8i+7 occupy 32 bytes; dims with (dim % 8) < 4 sit in the first 16, the
    // others in the last 16; vector v's nibble is in byte inv_perm[v % 16], low nibble for
    // v < 16, high nibble otherwise; its bit (3 - dim % 4) holds the sign bit.
    static const int perm[16] = {0, 8, 1, 9, 2, 10, 3, 11, 4, 12, 5, 13, 6, 14, 7, 15};
    int inv_perm[16];
    for (int j = 0; j < 16; ++j) inv_perm[perm[j]] = j;
    std::vector<uint8_t> batch, ex;
    auto read_at = [&](uint64_t at, void *dst, uint64_t bytes) {
        in.seekg(static_cast<std::streamoff>(at));
        in.read(reinterpret_cast<char *>(dst), static_cast<std::streamsize>(bytes));
        if (!in) fail(CORA_EINVAL, "Failed to read IVF index payload");
        f.bytes_read += bytes;
    };
    for (uint64_t c0 = 0; c0 < f.nlist;) {
        if (!f.owned[c0]) {
            ++c0;
            continue;
        }
        uint64_t c1 = c0;  // run [c0, c1) of consecutive owned clusters
        while (c1 < f.nlist && f.owned[c1]) ++c1;
        batch.resize((bstart[c1] - bstart[c0]) * rec);
        read_at(batch_at + bstart[c0] * rec, batch.data(), batch.size());
        const uint64_t rn = cstart[c1] - cstart[c0];
        ex.resize(rn * ex_stride);
        read_at(ex_at + cstart[c0] * ex_stride, ex.data(), ex.size());
        read_at(ids_at + cstart[c0] * 4, f.ids.data() + lstart[c0], rn * 4);
#pragma omp parallel for schedule(dynamic, 16)
        for (int64_t c = static_cast<int64_t>(c0); c < static_cast<int64_t>(c1); ++c) {
            const uint64_t n = full_sizes[c], s = lstart[c];
            for (uint64_t i = 0; i < n; i += 32) {
                const uint8_t *blk = batch.data() + (bstart[c] - bstart[c0] + i / 32) * rec;
                const float *fa = reinterpret_cast<const float *>(blk + D * 4);
                const uint64_t len = std::min<uint64_t>(32, n - i);
                for (uint64_t v = 0; v < len; ++v) {
                    for (uint64_t w = 0; w < W; ++w) {
                        uint32_t word = 0;
                        for (int b = 0; b < 32; ++b) {
                            const uint64_t d = w * 32 + b;
                            const uint8_t byte =
                                blk[(d / 8) * 32 + ((d % 8) < 4 ? 0 : 16) + inv_perm[v % 16]];
                            const uint8_t nib = v < 16 ? (byte & 0x0F) : (byte >> 4);
                            word |= static_cast<uint32_t>((nib >> (3 - (d % 4))) & 1u) << (31 - b);
                        }
                        f.short_data[s * W + w * n + i + v] = word;
                    }
                    for (int t = 0; t < 3; ++t)
                        f.short_factors[(s + i + v) * 3 + t] = fa[t * 32 + v];
                }
            }
            const uint64_t e0 = cstart[c] - cstart[c0];
            for (uint64_t i = 0; i < n; ++i) {
                std::memcpy(f.long_codes.data() + (s + i) * lc, ex.data() + (e0 + i) * ex_stride, lc);
                std::memcpy(f.ex_factors.data() + (s + i) * 2,
                            ex.data() + (e0 + i) * ex_stride + lc, 8);
            }
        }
        c0 = c1;
    }
    return f;
}
}  // namespace

}  // namespace cora

// ======================================================================================
// C ABI
// ======================================================================================
using cora::Engine;

struct cora_engine {
    std::unique_ptr<Engine> e;
};

namespace {
template <typename F>
int guarded(F &&f) {
    try {
        f();
        return CORA_OK;
    } catch (const cora::Error &e) {
        cora::g_last_error = e.what();
        return e.code;
    } catch (const std::bad_alloc &e) {
        cora::g_last_error = e.what();
        return CORA_ENOMEM;
    } catch (const std::exception &e) {
        cora::g_last_error = e.what();
        return CORA_ERUNTIME;
    }
}
Engine &eng(cora_engine *h) {
    if (!h || !h->e) cora::fail(CORA_EINVAL, "null engine");
    return *h->e;
}
const Engine &eng(const cora_engine *h) {
    if (!h || !h->e) cora::fail(CORA_EINVAL, "null engine");
    return *h->e;
}
}  // namespace

extern "C" {

const char *cora_last_error(void) { return cora::g_last_error.c_str(); }

int cora_create(cora_engine **out, int device) {
    return guarded([&] {
        if (!out) cora::fail(CORA_EINVAL, "null output handle");
        auto h = std::make_unique<cora_engine>();
        h->e = std::make_unique<Engine>(device);
        *out = h.release();
    });
}

void cora_destroy(cora_engine *engine) { delete engine; }

int cora_load_from_raw_pointers(cora_engine *engine, uint64_t num_vecs, uint64_t d, uint64_t p_d,
                                uint64_t n_centroids, uint64_t ex_b, const float *h_centroids,
                                const float *h_rotator, const uint32_t *h_short_data,
                                const float *h_short_factors, const uint8_t *h_long_code,
                                const float *h_ex_factors, const uint32_t *h_ids,
                                const uint64_t *h_cluster_sizes) {
    return guarded([&] {
        eng(engine).load_any(num_vecs, d, p_d, n_centroids, ex_b, h_centroids, h_rotator,
                             h_short_data, h_short_factors, h_long_code, h_ex_factors, h_ids,
                             h_cluster_sizes);
    });
}

int cora_load_index_file(cora_engine *engine, const char *path) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.loaded) cora::fail(CORA_ESTATE, "index already loaded");
        if (!path) cora::fail(CORA_EINVAL, "null index path");
        if (e.shard_world > 1) {  // read this shard's clusters only
            cora::FileIndex f = cora::read_index_file(path, e.shard_rank, e.shard_world);
            e.load_shard_local(f.num, f.dim, f.D, f.nlist, f.ex_bits, f.centroids.data(),
                               f.rotator.data(), f.short_data.data(), f.short_factors.data(),
                               f.long_codes.data(), f.ex_factors.data(), f.ids.data(),
                               f.sizes.data(), f.owned, f.kept);
            e.set_metric(f.metric);
            return;
        }
        cora::FileIndex f = cora::read_index_file(path);
        e.set_metric(f.metric);
        e.load_any(f.num, f.dim, f.D, f.nlist, f.ex_bits, f.centroids.data(), f.rotator.data(),
               f.short_data.data(), f.short_factors.data(), f.long_codes.data(), f.ex_factors.data(),
               f.ids.data(), f.sizes.data());
    });
}

int cora_index_file_shard_info(const char *path, uint32_t rank, uint32_t world,
                               uint64_t *out4) {
    return guarded([&] {
        if (!path || !out4) cora::fail(CORA_EINVAL, "null argument");
        if (world == 0 || world > cora::kMaxShards || rank >= world)
            cora::fail(CORA_EINVAL, "invalid shard rank / world");
        std::ifstream in(path, std::ios::binary);
        if (!in) cora::fail(CORA_EINVAL, std::string("Cannot open IVF index: ") + path);
        uint64_t hdr[4];
        uint8_t types[2];
        in.read(reinterpret_cast<char *>(hdr), sizeof(hdr));
        in.read(reinterpret_cast<char *>(types), 2);
        if (!in || !hdr[2] || !hdr[1]) cora::fail(CORA_EINVAL, "truncated IVF index header");
        const uint64_t nlist = hdr[2], D = (hdr[1] + 63) / 64 * 64;
        std::vector<uint64_t> sizes(nlist);
        in.read(reinterpret_cast<char *>(sizes.data()), 8 * nlist);
        if (!in) cora::fail(CORA_EINVAL, "truncated IVF index header");
        std::vector<int32_t> owner(nlist, 0);
        if (world > 1) cora::plan_shards(sizes.data(), nlist, world, owner.data());
        const uint64_t rec = D * 4 + 32 * 12, ex_stride = hdr[3] ? D * hdr[3] / 8 + 8 : 0;
        uint64_t vecs = 0, clusters = 0, bytes = 0;
        for (uint64_t c = 0; c < nlist; ++c)
            if (owner[c] == static_cast<int32_t>(rank)) {
                vecs += sizes[c];
                ++clusters;
                bytes += (sizes[c] + 31) / 32 * rec + sizes[c] * (ex_stride + 4);
            }
        out4[0] = vecs;
        out4[1] = clusters;
        out4[2] = bytes;
        out4[3] = hdr[0];
    });
}

int cora_index_info(const cora_engine *engine, uint64_t *out6) {
    return guarded([&] {
        const Engine &e = eng(engine);
        if (!e.loaded) cora::fail(CORA_ESTATE, "no index loaded");
        if (!out6) cora::fail(CORA_EINVAL, "null output");
        const uint64_t v[6] = {e.N, e.dim, e.D, e.nlist, e.ex_bits, e.max_cluster};
        std::memcpy(out6, v, sizeof(v));
    });
}

int cora_prepare_workspace(cora_engine *engine, uint64_t max_queries, uint64_t max_topk,
                           uint64_t max_nprobe) {
    return guarded([&] { eng(engine).prepare_workspace(max_queries, max_topk, max_nprobe); });
}

void cora_free_workspace(cora_engine *engine) {
    if (engine && engine->e) engine->e->free_workspace();
}

int cora_reset_buffer(cora_engine *engine, const float *h_queries, uint64_t num_queries) {
    return guarded([&] { eng(engine).reset_buffer(h_queries, num_queries); });
}

int cora_enable_exact_refine(cora_engine *engine, const uint8_t *base_mapping,
                             uint64_t base_rows, uint64_t base_dim, uint64_t row_stride_bytes,
                             uint64_t data_offset_bytes) {
    return guarded([&] {
        Engine &e = eng(engine);
        CUDA_TRY(cudaSetDevice(e.device));
        e.enable_exact_refine(base_mapping, base_rows, base_dim, row_stride_bytes,
                              data_offset_bytes);
    });
}

int cora_search(cora_engine *engine, const float *h_queries, uint64_t num_queries, uint64_t topk,
                uint64_t nprobe, float *h_final_dists, uint32_t *h_final_pids, int batch_q) {
    return guarded([&] {
        eng(engine).search_host(h_queries, num_queries, topk, nprobe, h_final_dists, h_final_pids,
                                batch_q);
    });
}

int cora_search_device(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                       uint64_t topk, uint64_t nprobe, float *d_final_dists,
                       uint32_t *d_final_pids, void *stream) {
    return guarded([&] {
        Engine &e = eng(engine);
        e.validate_ws(num_queries, topk, nprobe);
        e.require_whole_index();
        if (!d_queries || !d_final_dists || !d_final_pids)
            cora::fail(CORA_EINVAL, "invalid device search buffers");
        CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e.stream;
        e.enqueue_search(d_queries, num_queries, topk, nprobe, d_final_dists, d_final_pids, st);
    });
}

// ---- cluster-sharded search ---------------------------------------------------------------
int cora_shard_plan(const uint64_t *sizes, uint64_t nlist, uint32_t world, int32_t *owner_out) {
    return guarded([&] {
        if (!sizes || !owner_out || nlist == 0 || world == 0 || world > cora::kMaxShards)
            cora::fail(CORA_EINVAL, "invalid shard plan arguments");
        cora::plan_shards(sizes, nlist, world, owner_out);
    });
}

int cora_shard_configure(cora_engine *engine, uint32_t rank, uint32_t world) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.loaded) cora::fail(CORA_ESTATE, "configure sharding before loading the index");
        if (world == 0 || world > cora::kMaxShards || rank >= world)
            cora::fail(CORA_EINVAL, "shard rank must be in [0, world) and world in [1, 256]");
        e.shard_rank = rank;
        e.shard_world = world;
    });
}

int cora_load_shard_arrays(cora_engine *engine, uint64_t local_vecs, uint64_t d, uint64_t p_d,
                           uint64_t n_centroids, uint64_t ex_b, const float *h_centroids,
                           const float *h_rotator, const uint32_t *h_short_data,
                           const float *h_short_factors, const uint8_t *h_long_code,
                           const float *h_ex_factors, const uint32_t *h_ids,
                           const uint64_t *h_local_sizes, const uint64_t *h_global_sizes) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.loaded) cora::fail(CORA_ESTATE, "index already loaded");
        if (!h_local_sizes || !h_global_sizes || n_centroids == 0)
            cora::fail(CORA_EINVAL, "null cluster sizes");
        std::vector<int32_t> owner(n_centroids, 0);
        if (e.shard_world > 1)
            cora::plan_shards(h_global_sizes, n_centroids, e.shard_world, owner.data());
        std::vector<uint8_t> mask(n_centroids, 0);
        uint64_t local = 0, kept = 0;
        for (uint64_t c = 0; c < n_centroids; ++c) {
            const bool own = owner[c] == static_cast<int32_t>(e.shard_rank);
            if (h_local_sizes[c] != (own ? h_global_sizes[c] : 0))
                cora::fail(CORA_EINVAL, "cluster " + std::to_string(c) +
                                            ": local size differs from this shard's plan");
            if (own) {
                mask[c] = 1;
                local += h_global_sizes[c];
                ++kept;
            }
        }
        if (local != local_vecs) cora::fail(CORA_EINVAL, "local cluster sizes differ from local_vecs");
        if (e.shard_world <= 1) {
            e.load_any(local_vecs, d, p_d, n_centroids, ex_b, h_centroids, h_rotator, h_short_data,
                       h_short_factors, h_long_code, h_ex_factors, h_ids, h_local_sizes);
            return;
        }
        e.load_shard_local(local_vecs, d, p_d, n_centroids, ex_b, h_centroids, h_rotator,
                           h_short_data, h_short_factors, h_long_code, h_ex_factors, h_ids,
                           h_local_sizes, mask, kept);
    });
}

int cora_shard_info(const cora_engine *engine, uint64_t *out4) {
    return guarded([&] {
        const Engine &e = eng(engine);
        if (!out4) cora::fail(CORA_EINVAL, "null output");
        out4[0] = e.shard_rank;
        out4[1] = e.shard_world;
        out4[2] = e.loaded ? e.N : 0;
        out4[3] = e.loaded ? e.shard_clusters : 0;
    });
}

uint64_t cora_shard_exchange_words(uint64_t num_queries, uint64_t topk) {
    return Engine::exchange_stride(num_queries, topk);
}

int cora_shard_search_begin(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                            uint64_t topk, uint64_t nprobe, uint64_t *d_send, void *stream) {
    return guarded([&] {
        Engine &e = eng(engine);
        e.validate_ws(num_queries, topk, nprobe);
        if (!d_queries || !d_send) cora::fail(CORA_EINVAL, "invalid device search buffers");
        CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e.stream;
        e.split_phase = 0;
        e.enqueue_front(d_queries, num_queries, topk, nprobe, st, d_send);
        e.split_phase = 1;
    });
}

uint64_t cora_shard_probe_words(uint64_t num_queries, uint64_t nprobe, uint32_t world) {
    if (world == 0) return 0;
    return (num_queries + world - 1) / world * nprobe + 1;
}

int cora_shard_search_probe(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                            uint64_t topk, uint64_t nprobe, uint64_t *d_send, void *stream) {
    return guarded([&] {
        Engine &e = eng(engine);
        e.validate_ws(num_queries, topk, nprobe);
        if (!d_queries || !d_send) cora::fail(CORA_EINVAL, "invalid device search buffers");
        if (e.shard_world > 256) cora::fail(CORA_EINVAL, "at most 256 shards");
        CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e.stream;
        e.split_phase = 0;
        const uint64_t world = e.shard_world, slice = (num_queries + world - 1) / world;
        const uint64_t q0 = std::min<uint64_t>(num_queries, e.shard_rank * slice);
        const uint64_t q1 = std::min<uint64_t>(num_queries, q0 + slice);
        e.enqueue_rotate(d_queries, num_queries, topk, nprobe, st);
        e.enqueue_probe_range(q0, q1, st);
        const uint64_t stride = cora_shard_probe_words(num_queries, nprobe, e.shard_world);
        const size_t n = (q1 - q0) * nprobe;
        cora::pack_probes_kernel<<<static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(
                                       (n + 255) / 256, 4 * (size_t)e.num_sms))),
                                   256, 0, st>>>(e.probe_ids.p + q0 * nprobe,
                                                 e.probe_g.p + q0 * nprobe, n, e.err.p, d_send,
                                                 stride);
        CUDA_TRY(cudaGetLastError());
        e.split_phase = 3;
    });
}

int cora_shard_search_begin_probed(cora_engine *engine, const uint64_t *d_recv,
                                   uint64_t *d_send) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.split_phase != 3) cora::fail(CORA_ESTATE, "shard search: probe must come first");
        if (!d_recv || !d_send) cora::fail(CORA_EINVAL, "invalid exchange buffers");
        CUDA_TRY(cudaSetDevice(e.device));
        e.split_phase = 0;
        cudaStream_t st = e.last_stream;
        const uint64_t nq = e.last_nq, np = e.last_np, world = e.shard_world;
        const uint64_t slice = (nq + world - 1) / world;
        cora::unpack_probes_kernel<<<static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>(
                                         (nq * np + 255) / 256, 4 * (uint64_t)e.num_sms))),
                                     256, 0, st>>>(d_recv, static_cast<int>(world),
                                                   cora_shard_probe_words(nq, np, e.shard_world),
                                                   slice, nq, static_cast<int>(np), e.probe_ids.p,
                                                   e.probe_g.p, e.err.p);
        CUDA_TRY(cudaGetLastError());
        e.enqueue_probe_gadd(st);
        e.mark(3, st);
        e.enqueue_vanguard(d_send);
        e.split_phase = 1;
    });
}

int cora_shard_search_resume(cora_engine *engine, const uint64_t *d_recv, uint64_t *d_send) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.split_phase != 1) cora::fail(CORA_ESTATE, "shard search: begin must come first");
        if (!d_recv || !d_send) cora::fail(CORA_EINVAL, "invalid exchange buffers");
        CUDA_TRY(cudaSetDevice(e.device));
        e.split_phase = 0;
        e.enqueue_back(d_recv, static_cast<int>(e.shard_world), nullptr, nullptr, d_send);
        e.split_phase = 2;
    });
}

int cora_shard_search_end(cora_engine *engine, const uint64_t *d_recv, float *d_final_dists,
                          uint32_t *d_final_pids) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.split_phase != 2) cora::fail(CORA_ESTATE, "shard search: resume must come first");
        if (!d_recv || !d_final_dists || !d_final_pids)
            cora::fail(CORA_EINVAL, "invalid exchange or result buffers");
        CUDA_TRY(cudaSetDevice(e.device));
        e.split_phase = 0;
        e.enqueue_final(d_recv, static_cast<int>(e.shard_world), d_final_dists, d_final_pids);
    });
}

int cora_check_device(cora_engine *engine) {
    return guarded([&] {
        Engine &e = eng(engine);
        e.require_ws();
        CUDA_TRY(cudaSetDevice(e.device));
        e.finish(e.last_stream);
    });
}

int cora_seed_thresholds(cora_engine *engine, const float *h_in, uint64_t nq) {
    return guarded([&] { eng(engine).seed_thresholds(h_in, nq); });
}

int cora_capture_thresholds(const cora_engine *engine, float *h_out, uint64_t nq) {
    return guarded([&] { eng(engine).capture_thresholds(h_out, nq); });
}

int cora_set_vanguard_size(cora_engine *engine, uint64_t size) {
    return guarded([&] { eng(engine).set_vanguard(size); });
}
uint64_t cora_get_vanguard_size(const cora_engine *engine) {
    return engine && engine->e ? engine->e->vanguard : 0;
}

// hybrid.cu:166-185
int cora_set_queue_capacity(cora_engine *engine, uint64_t capacity) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (capacity == 0 || (capacity & (capacity - 1)) != 0 || capacity > (SIZE_MAX >> 5))
            cora::fail(CORA_EINVAL, "queue-capacity must be a positive power of two");
        if (e.ws_ready) cora::fail(CORA_ESTATE, "set queue capacity before prepare_workspace");
        e.queue_capacity = capacity;
    });
}
int cora_set_queue_spill_capacity(cora_engine *engine, uint64_t capacity) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (capacity > (SIZE_MAX >> 5)) cora::fail(CORA_EINVAL, "queue-spill-capacity is too large");
        if (e.ws_ready) cora::fail(CORA_ESTATE, "set spill capacity before prepare_workspace");
        e.spill_capacity = capacity;
    });
}
uint64_t cora_get_queue_capacity(const cora_engine *engine) {
    return engine && engine->e ? engine->e->queue_capacity : 0;
}

void cora_set_profiling(cora_engine *engine, int enabled) {
    if (engine && engine->e) engine->e->profiling = enabled != 0;
}
void cora_set_candidate_stats(cora_engine *engine, int enabled) {
    if (engine && engine->e) engine->e->candidate_stats = enabled != 0;
}
void cora_set_gpu_filter_timing(cora_engine *engine, int enabled) {
    if (engine && engine->e) engine->e->gpu_filter_timing = enabled != 0;
}
void cora_set_cross_query_reuse(cora_engine *engine, int enabled) {
    if (engine && engine->e) engine->e->cross_query_reuse = enabled != 0;
}
void cora_set_cpu_secondary_filter(cora_engine *engine, int enabled) {
    if (engine && engine->e) engine->e->cpu_secondary_filter = enabled != 0;
}
void cora_set_ip_kernel_type(cora_engine *engine, int kernel_type) {
    if (engine && engine->e) engine->e->ip_kernel_type = kernel_type == 0 ? 0 : 1;
}
int cora_get_ip_kernel_type(const cora_engine *engine) {
    return engine && engine->e ? engine->e->ip_kernel_type : 0;
}
int cora_set_metric(cora_engine *engine, int metric) {
    return guarded([&] { eng(engine).set_metric(metric); });
}
int cora_get_metric(const cora_engine *engine) {
    return engine && engine->e ? engine->e->metric : -1;
}
void cora_set_refine_full_code(cora_engine *engine, int enabled) {
    if (engine && engine->e) engine->e->refine_full_code = enabled != 0;
}
int cora_get_refine_full_code(const cora_engine *engine) {
    return engine && engine->e ? (engine->e->refine_full_code ? 1 : 0) : 0;
}

uint64_t cora_get_last_submitted_count(const cora_engine *engine) {
    return engine && engine->e ? engine->e->last_submitted : 0;
}
uint64_t cora_get_last_refined_count(const cora_engine *engine) {
    return engine && engine->e ? engine->e->last_refined : 0;
}
uint64_t cora_get_last_spilled_count(const cora_engine *) { return 0; }
float cora_get_last_gpu_filter_ms(const cora_engine *engine) {
    return engine && engine->e ? engine->e->last_filter_ms : 0.0f;
}

int cora_debug_copy(cora_engine *engine, int what, void *h_out, uint64_t bytes) {
    return guarded([&] {
        if (!h_out) cora::fail(CORA_EINVAL, "null output");
        eng(engine).debug_copy(what, h_out, bytes);
    });
}

int cora_get_last_stage_ms(cora_engine *engine, float *h_out, uint64_t n) {
    return guarded([&] {
        if (!h_out) cora::fail(CORA_EINVAL, "null output");
        Engine &e = eng(engine);
        CUDA_TRY(cudaSetDevice(e.device));
        e.stage_ms(h_out, n);
    });
}

int cora_stage_totals(cora_engine *engine, double *h_out, uint64_t n, uint64_t *h_count) {
    return guarded([&] {
        if (!h_out || !h_count) cora::fail(CORA_EINVAL, "null output");
        Engine &e = eng(engine);
        CUDA_TRY(cudaSetDevice(e.device));
        *h_count = e.stage_totals(h_out, n);
    });
}

int cora_stage_reset(cora_engine *engine) {
    return guarded([&] { eng(engine).stage_reset(); });
}

int cora_set_vanguard_lows_budget(cora_engine *engine, uint64_t bytes) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (e.ws_ready) cora::fail(CORA_ESTATE, "set the lows budget before prepare_workspace");
        e.lows_budget = bytes;
    });
}

int cora_set_tuning(cora_engine *engine, const char *key, int64_t value) {
    return guarded([&] {
        Engine &e = eng(engine);
        const std::string k = key ? key : "";
        if (k == "warp_select_limit") {
            if (value < 0 || value > cora::kWarpSelectBuf)
                cora::fail(CORA_EINVAL, "warp_select_limit must be in [0, 256]");
            e.warp_select_limit = static_cast<int>(value);
        } else if (k == "topk_warp_limit") {
            if (value < 0 || value > cora::kWarpTopBuf)
                cora::fail(CORA_EINVAL, "topk_warp_limit must be in [0, 256]");
            e.topk_warp_limit = static_cast<int>(value);
        } else if (k == "refine_lanes") {
            if (value != 0 && value != 1 && value != 4 && value != 8)
                cora::fail(CORA_EINVAL, "refine_lanes must be 0, 1, 4 or 8");
            e.refine_lanes = static_cast<int>(value);
        } else if (k == "vanguard_lows_budget") {
            if (value < 0) cora::fail(CORA_EINVAL, "vanguard_lows_budget must be >= 0");
            if (e.ws_ready) cora::fail(CORA_ESTATE, "set the lows budget before prepare_workspace");
            e.lows_budget = static_cast<uint64_t>(value);
        } else if (k == "search_graphs") {
            if (value != 0 && value != 1) cora::fail(CORA_EINVAL, "search_graphs must be 0 or 1");
            e.search_graphs = value != 0;
            if (!e.search_graphs) e.drop_graph();
        } else {
            cora::fail(CORA_EINVAL, "unknown tuning key: " + k);
        }
    });
}

int cora_get_vanguard_mode(const cora_engine *engine) {
    return engine && engine->e ? (engine->e->lows.n > 0 ? 1 : 0) : -1;
}

uint64_t cora_get_candidate_capacity(const cora_engine *engine) {
    return engine && engine->e ? engine->e->cap : 0;
}

}  // extern "C"

// ======================================================================================
// Coarse probing without allocation (cora_probe_noalloc)
//
// Some callers cannot allocate device memory at the point where they need the probe list:
// a router that decides which GPU or shard owns a query's clusters before the search is
// dispatched, running next to searches it must not stall (cudaMalloc/cudaFree synchronise
// the device), or a process that cannot afford the multi-GB search workspace that
// prepare_workspace reserves. For them this entry point runs the same rotation, approximate
// distance and guarded top-nprobe kernels as a search, but keeps every intermediate in one
// fixed block of device memory that is part of the loaded module, so the call itself never
// allocates: no cudaMalloc/cudaFree, no library routine that allocates, no host buffer on
// the success path (a rejected call only builds its error message).
//
// Limits and rules:
//  * the scratch block is kNoallocScratchBytes (16 MiB) per device; a call needing more
//    (num_queries * per-query bytes, see noalloc_scratch_bytes) is rejected with
//    CORA_EINVAL and a message giving both sizes;
//  * nothing in the block has to start at zero: every kernel writes each scratch element
//    before any kernel reads it;
//  * the first call on a device, with that device current, looks the block's address up
//    (cudaGetSymbolAddress) and caches it with the device's current context; make that first
//    call before any stream capture. After the context is torn down and created again
//    (cudaDeviceReset), the next call looks the address up again, so it too must come before
//    any capture;
//  * there is ONE block per device, shared by every engine on that device: calls that
//    overlap in time (two streams, two host threads) race on it and corrupt each other's
//    results. Serialise them, e.g. issue them all on one stream.
// ======================================================================================
namespace cora {
namespace {

constexpr size_t kNoallocScratchBytes = size_t{16} << 20;
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mutex;
// Per device: the context the address was looked up in, and the address. A context that is
// torn down and created again (cudaDeviceReset) loads the module anew, so the address is
// looked up again whenever the device's current context differs from the cached one.
struct NoallocSlot {
    void *ctx = nullptr;
    unsigned char *ptr = nullptr;
};
NoallocSlot g_noalloc_slot[kNoallocMaxDevices];

using CtxGetCurrentFn = int (*)(void **);
inline void *current_context() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    });
    if (!fn) fail(CORA_ECUDA, "the driver does not provide cuCtxGetCurrent");
    void *ctx = nullptr;
    if (fn(&ctx) != 0 || !ctx) fail(CORA_ECUDA, "no current CUDA context");
    return ctx;
}

inline size_t align256(size_t b) { return (b + 255) & ~size_t{255}; }

struct NoallocLayout {
    size_t status, qr, qnorm2, scal, planes, approx, chunk_min, fallback, total;
};

NoallocLayout noalloc_layout(uint64_t nq, uint64_t D, uint64_t W4, uint64_t nlist) {
    NoallocLayout l{};
    l.status = 0;  // device error word of the last call (zeroed by each call)
    l.qr = 256;
    l.qnorm2 = l.qr + align256(nq * D * sizeof(float));
    l.scal = l.qnorm2 + align256(nq * sizeof(float));
    l.planes = l.scal + align256(nq * sizeof(QueryScalars));
    l.approx = l.planes + align256(nq * 8 * W4 * sizeof(uint32_t));
    l.chunk_min = l.approx + align256(nq * approx_ld(nlist) * sizeof(float));
    l.fallback = l.chunk_min + align256(nq * chunk_stride(static_cast<int>(nlist)) * sizeof(float));
    l.total = l.fallback + align256((nq + 1) * sizeof(uint32_t));
    return l;
}

// Address of this device's scratch block in its current context; the device must be current.
unsigned char *noalloc_scratch(int device) {
    if (device < 0 || device >= kNoallocMaxDevices) fail(CORA_EINVAL, "device ordinal out of range");
    void *ctx = current_context();
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    NoallocSlot &slot = g_noalloc_slot[device];
    if (!slot.ptr || slot.ctx != ctx) {
        void *p = nullptr;
        const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (rc != cudaSuccess || !p)
            fail(CORA_ERUNTIME, std::string("cudaGetSymbolAddress for the probe scratch failed: ") +
                                    cudaGetErrorString(rc));
        slot.ctx = ctx;
        slot.ptr = static_cast<unsigned char *>(p);
    }
    return slot.ptr;
}

}  // namespace
}  // namespace cora

extern "C" {

uint64_t cora_probe_noalloc_scratch_limit(void) { return cora::kNoallocScratchBytes; }

int cora_probe_noalloc(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                       uint64_t nprobe, int32_t *d_probe_ids, float *d_probe_dists, void *stream) {
    return guarded([&] {
        Engine &e = eng(engine);
        if (!e.loaded) cora::fail(CORA_ESTATE, "load an index before probing");
        if (!d_queries || !d_probe_ids || !d_probe_dists)
            cora::fail(CORA_EINVAL, "invalid device probe buffers");
        if (num_queries == 0 || num_queries > cora::kMaxQueryChunk)
            cora::fail(CORA_EINVAL, "query count must be in [1, 65535]");
        if (nprobe == 0 || nprobe > e.nlist || nprobe > cora::kMaxProbeFast)
            cora::fail(CORA_EINVAL, "nprobe must be in [1, min(nlist, 4096)]");
        const cora::NoallocLayout l = cora::noalloc_layout(num_queries, e.D, e.W4, e.nlist);
        if (l.total > cora::kNoallocScratchBytes)
            cora::fail(CORA_EINVAL, "probe needs " + std::to_string(l.total) +
                                        " bytes of scratch; the static limit is " +
                                        std::to_string(cora::kNoallocScratchBytes) +
                                        " bytes: split the queries into smaller calls");
        CUDA_TRY(cudaSetDevice(e.device));
        unsigned char *s = cora::noalloc_scratch(e.device);
        float *qr = reinterpret_cast<float *>(s + l.qr);
        float *qnorm2 = reinterpret_cast<float *>(s + l.qnorm2);
        auto *scal = reinterpret_cast<cora::QueryScalars *>(s + l.scal);
        uint32_t *planes = reinterpret_cast<uint32_t *>(s + l.planes);
        float *approx = reinterpret_cast<float *>(s + l.approx);
        int *status = reinterpret_cast<int *>(s + l.status);
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e.stream;
        CUDA_TRY(cudaMemsetAsync(status, 0, sizeof(int), st));

        const float c_b = -static_cast<float>((1u << (e.ex_bits + 1)) - 1u) / 2.0f;
        cora::launch_rotate_prep(d_queries, num_queries, e.dim, e.D, e.W4, e.rotator.p, c_b, qr,
                                 scal, planes, qnorm2, nullptr, st);
        float *cmin = reinterpret_cast<float *>(s + l.chunk_min);
        cora::launch_probe_gemm(qr, qnorm2, num_queries, e.D, e.centroids.p, e.cnorm2.p, e.nlist,
                                approx, cmin, e.num_sms, st, status);
        cora::launch_guarded_select(approx, cmin, e.nlist, num_queries, nprobe, qr, qnorm2,
                                    e.centroids.p, e.cmax, e.D, d_probe_ids, d_probe_dists,
                                    reinterpret_cast<uint32_t *>(s + l.fallback), e.num_sms, st);
    });
}

int cora_probe_noalloc_status(cora_engine *engine, void *stream) {
    return guarded([&] {
        Engine &e = eng(engine);
        CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : e.stream;
        unsigned char *s = cora::noalloc_scratch(e.device);
        int h = 0;
        CUDA_TRY(cudaMemcpyAsync(&h, s, sizeof(int), cudaMemcpyDeviceToHost, st));
        CUDA_TRY(cudaStreamSynchronize(st));
        if (h & cora::kDevWaitTimeout) cora::fail(CORA_ERUNTIME, "a device-side wait timed out");
        if (h) cora::fail(CORA_ERUNTIME, "device reported an error");
    });
}

}  // extern "C"
