/*
 * cora_b200 — C ABI of the B200-native IVF-RaBitQ search engine (libcoraanns_b200.so).
 *
 * This is the drop-in boundary for the search hot path of CoraANNS. Every entry point
 * replaces one method of the reference's coraanns::HybridIndex
 * (include/coraanns/search/hybrid.cuh of the reference project); the line cited beside
 * each declaration is the method it replaces. The header-only C++ shim
 * cgcl-coraanns_b200/include/coraanns/search/hybrid.hpp wraps these functions back into
 * a class with the reference's exact method signatures and exception types.
 *
 * Conventions
 *  - plain pointers and sizes only; "h_" pointers are host memory, "d_" pointers device
 *    memory of the engine's device;
 *  - every function returning int returns a cora_status; on failure
 *    cora_last_error() (thread-local) holds the message;
 *  - one engine serves one search at a time (the reference's rule); calls are blocking
 *    unless stated otherwise;
 *  - results are row-major nq x topk, ascending by (distance, id), padded with
 *    (FLT_MAX, 0); ids are the original vector ids of the index.
 */
#ifndef CORA_B200_H
#define CORA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; the shim maps them to the reference's exception types. */
typedef enum {
    CORA_OK = 0,
    CORA_EINVAL = 1,   /* std::invalid_argument */
    CORA_ESTATE = 2,   /* std::logic_error */
    CORA_ERUNTIME = 3, /* std::runtime_error (e.g. candidate capacity exhausted) */
    CORA_ECUDA = 4,    /* std::runtime_error from a CUDA call */
    CORA_ENOMEM = 5    /* std::bad_alloc */
} cora_status;

typedef struct cora_engine cora_engine;

/* Thread-local message of the last failing call on this thread. */
const char *cora_last_error(void);

/* HybridIndex() (hybrid.cuh:116): binds `device`, creates the engine's stream. */
int cora_create(cora_engine **out, int device);
/* ~HybridIndex() (hybrid.cuh:119): releases every device resource. NULL is a no-op. */
void cora_destroy(cora_engine *engine);

/* load_from_raw_pointers (hybrid.cuh:186-190). Same argument meaning, with size_t*
 * cluster sizes passed as uint64_t*. Validation as hybrid.cu:107-121 (num <= UINT32_MAX,
 * p_d % 64 == 0, p_d >= d, ex_b <= 8, sizes sum to num; CORA_ESTATE if already loaded),
 * plus this engine's limits: ex_b == 7 and p_d <= 1024. Unlike the reference, the
 * extended codes, factors and ids are copied to HBM, so the host arrays need only live
 * for the duration of the call. */
int cora_load_from_raw_pointers(cora_engine *engine, uint64_t num_vecs, uint64_t d, uint64_t p_d,
                                uint64_t n_centroids, uint64_t ex_b, const float *h_centroids,
                                const float *h_rotator, const uint32_t *h_short_data,
                                const float *h_short_factors, const uint8_t *h_long_code,
                                const float *h_ex_factors, const uint32_t *h_ids,
                                const uint64_t *h_cluster_sizes);

/* IVF::load (third_party/rabitq/.../index/ivf/ivf.hpp:447-539) + index::SearchData
 * (src/index/search_data.cpp:9-127) + load_from_raw_pointers in one call: reads an
 * IVF-RaBitQ index file with embedded (flat) centroids and a matrix rotator. */
int cora_load_index_file(cora_engine *engine, const char *path);

/* Index shape after loading: out[0..5] = num, dim, padded_dim, nlist, ex_bits,
 * largest cluster size. */
int cora_index_info(const cora_engine *engine, uint64_t *out6);
/* A shard's share of an index file (no GPU needed): out4 = {vectors, clusters, payload
 * bytes, the file's total vectors} that shard `rank` of `world` (cora_shard_plan) holds and
 * reads. A shard engine's cora_load_index_file reads only those payload bytes (plus the
 * header, rotator and every centroid). */
int cora_index_file_shard_info(const char *path, uint32_t rank, uint32_t world, uint64_t *out4);

/* prepare_workspace (hybrid.cuh:167): validate_search_shape (parameters.hpp:15-25),
 * CORA_ESTATE without an index; frees and reallocates. */
int cora_prepare_workspace(cora_engine *engine, uint64_t max_queries, uint64_t max_topk,
                           uint64_t max_nprobe);
/* free_workspace (hybrid.cuh:168): idempotent. */
void cora_free_workspace(cora_engine *engine);
/* reset_buffer (hybrid.cuh:169): stages queries and resets every threshold to FLT_MAX;
 * CORA_ESTATE without a workspace, CORA_EINVAL if num_queries exceeds it. */
int cora_reset_buffer(cora_engine *engine, const float *h_queries, uint64_t num_queries);

/* enable_exact_refine (hybrid.cuh:171-178): refine candidates with the exact squared L2
 * distance between the raw query and base row `id` (the vector's original id), row id at
 * base_mapping + data_offset_bytes + id * row_stride_bytes, base_dim fp32 values; the
 * distance is the fp32 rounding of the fp64 fma chain over the dimensions ascending.
 * Candidates whose id >= base_rows, or every candidate when base_dim differs from the
 * index dimension, are dropped (cpu_refinement.cpp:168-181). The rows this engine holds are
 * copied into HBM now (or when the index is loaded), so the mapping must stay valid until
 * then. base_mapping == NULL turns exact refinement off. CORA_EINVAL when the stride is
 * shorter than a row. */
int cora_enable_exact_refine(cora_engine *engine, const uint8_t *base_mapping,
                             uint64_t base_rows, uint64_t base_dim, uint64_t row_stride_bytes,
                             uint64_t data_offset_bytes);

/* search (hybrid.cuh:195-196): blocking; CORA_EINVAL unless 1 <= batch_q <= 6 or if the
 * shape exceeds the workspace; CORA_ERUNTIME with "spill capacity exhausted" when the
 * per-query candidate capacity ((queue + spill capacity) / max_queries) overflows. */
int cora_search(cora_engine *engine, const float *h_queries, uint64_t num_queries,
                uint64_t topk, uint64_t nprobe, float *h_final_dists, uint32_t *h_final_pids,
                int batch_q);

/* Device-resident variant of search (no reference counterpart; used by multi-GPU
 * callers and for kernel-only timing): queries, outputs in device memory, enqueued on
 * `stream` (a cudaStream_t, NULL for the engine's own stream); returns without
 * synchronising. Errors raised on the device are reported by cora_check_device(). */
int cora_search_device(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                       uint64_t topk, uint64_t nprobe, float *d_final_dists,
                       uint32_t *d_final_pids, void *stream);
/* Synchronises the engine's last stream and turns device-side error flags into a status. */
int cora_check_device(cora_engine *engine);

/* seed_thresholds / capture_thresholds (hybrid.cuh:192-193). */
int cora_seed_thresholds(cora_engine *engine, const float *h_in, uint64_t nq);
int cora_capture_thresholds(const cora_engine *engine, float *h_out, uint64_t nq);

/* set_vanguard_size / get_vanguard_size (hybrid.cuh:155-158): CORA_ESTATE when raising
 * the depth above the one the workspace was prepared for (hybrid.cu:87-91). */
int cora_set_vanguard_size(cora_engine *engine, uint64_t size);
uint64_t cora_get_vanguard_size(const cora_engine *engine);

/* set_queue_capacity / set_queue_spill_capacity / get_queue_capacity
 * (hybrid.cuh:143-147, validation hybrid.cu:166-185). Their sum bounds the candidate
 * records held in HBM per search. */
int cora_set_queue_capacity(cora_engine *engine, uint64_t capacity);
int cora_set_queue_spill_capacity(cora_engine *engine, uint64_t capacity);
uint64_t cora_get_queue_capacity(const cora_engine *engine);

/* Knobs (hybrid.cuh:121-135,160-165). cross_query_reuse=0 processes one query per
 * cluster work item; cpu_secondary_filter is accepted for drop-in compatibility (refinement
 * runs on the GPU). ip_kernel_type selects the scan's estimator (hybrid.cuh:12):
 * 0 = Lut4Bit, ip1 from fp16 lookup tables of the rotated query (query_kernels.cuh:199-221,
 * filter_kernels.cuh:283-306), the reference's default; 1 = Bitwise, ip1 = width * ip_int
 * from the integer estimator (filter_kernels.cuh:79-114), THIS ENGINE'S DEFAULT (exact
 * integer arithmetic, the fastest scan). Any other value selects Bitwise. Both feed the same
 * lower bound and refinement expression. */
void cora_set_profiling(cora_engine *engine, int enabled);
void cora_set_candidate_stats(cora_engine *engine, int enabled);
void cora_set_gpu_filter_timing(cora_engine *engine, int enabled);
void cora_set_cross_query_reuse(cora_engine *engine, int enabled);
void cora_set_cpu_secondary_filter(cora_engine *engine, int enabled);
void cora_set_ip_kernel_type(cora_engine *engine, int kernel_type);
int cora_get_ip_kernel_type(const cora_engine *engine);

/* Distance of the index (no counterpart in the reference's hybrid path, which is L2 only;
 * the reference's CPU path supports both, ivf.hpp:681-706): 0 squared L2 (default), 1 inner
 * product, where distances are the reference IP factors' estimates of 1 - <q, x> and the
 * additive query term is -<q', c'> (index/query.hpp:99-108; probes stay the nearest centroids
 * by L2 distance). cora_load_index_file sets it from the file header's MetricType; indexes
 * loaded from raw arrays must be built for the metric set here. CORA_EINVAL for other values
 * or for inner product with exact refinement enabled. Takes effect from the next search.
 * cora_get_metric returns -1 for a NULL engine. */
int cora_set_metric(cora_engine *engine, int metric);
int cora_get_metric(const cora_engine *engine);

/* Refinement form (no reference counterpart; the reference always uses its default).
 * 0 (default): the reference's expression, ex = (f_add_ex + g) + f_rescale_ex *
 * ((128 ip1 + ip2) + kb), ip1 = width * ip_int the scan's integer estimate of <q', b>
 * (cpu_refinement.cpp:183-191). 1: the full 8-bit code inner product <q', 128 b + u> in place
 * of 128 ip1 + ip2, which removes the query-quantisation error of ip1 (better recall; results
 * then differ from the reference's). Takes effect from the next search. */
void cora_set_refine_full_code(cora_engine *engine, int enabled);
int cora_get_refine_full_code(const cora_engine *engine);

/* Counters of the last search (hybrid.cuh:137-153). submitted = candidates that passed
 * the 1-bit lower bound (seeds included); refined = candidates refined with ex codes;
 * spilled is always 0 (no host ring). */
uint64_t cora_get_last_submitted_count(const cora_engine *engine);
uint64_t cora_get_last_refined_count(const cora_engine *engine);
uint64_t cora_get_last_spilled_count(const cora_engine *engine);
float cora_get_last_gpu_filter_ms(const cora_engine *engine);

/* Diagnostics for parity tests (no reference counterpart): copies an intermediate of
 * the last search to host memory. what: 0 rotated queries (nq x D f32), 1 probe ids
 * (nq x nprobe i32), 2 probe distances (nq x nprobe f32), 3 per-query candidate counts
 * (nq u32), 4 thresholds after seeding (nq f32), 5 query bit-planes
 * (nq x 8 x W4 u32, W4 = 4 * ceil(D / 128)), 6 query scalars (nq x {width, k1, kb, sumq}),
 * 7 candidate gids (nq x cap u32, per query sorted ascending, unused slots 0xFFFFFFFF),
 * 8 approximate coarse distances of the tensor-core probe GEMM (nq x ld f32, ld = nlist
 * rounded up to a multiple of 4; rows the exact fallback recomputed hold exact values),
 * 9 LUT estimator tables (nq x D/4 x 16 binary16; written only with kernel type Lut4Bit),
 * 10 the estimator's additive query term g_add per probe (nq x nprobe f32; = array 2 for L2,
 * -<q', c'> for inner product).
 * `bytes` must equal the size of the requested array. */
int cora_debug_copy(cora_engine *engine, int what, void *h_out, uint64_t bytes);
/* Per-stage device times (ms) of the last search run with profiling enabled, from CUDA
 * events recorded between the launches on the search stream: 0 rotation + query prep,
 * 1 coarse distances, 2 top-nprobe, 3 vanguard pair grouping, 4 vanguard scan (lows pass
 * or rescan), 5 vanguard seed selection, 6 seed refine, 7 threshold, 8 main pair grouping,
 * 9 main scan, 10 vanguard lows filter, 11 main refine, 12 merge. Writes min(n, 13). */
int cora_get_last_stage_ms(cora_engine *engine, float *h_out, uint64_t n);
/* Sums of the same per-stage times over every profiled search since cora_stage_reset();
 * *h_count receives the number of searches summed. Reading never stalls searches that are
 * still queued: each search's events are read back when its slot in a 16-entry ring is
 * reused, or here. */
int cora_stage_totals(cora_engine *engine, double *h_out, uint64_t n, uint64_t *h_count);
int cora_stage_reset(cora_engine *engine);
/* Budget (bytes, default 16 GiB, capped at a quarter of free HBM) of the buffer that keeps
 * the vanguard pairs' 1-bit lower bounds between the seeding and main passes, so that the
 * vanguard clusters are scanned once. prepare_workspace sizes it for the worst case
 * (every query probing the largest clusters); above the budget the vanguard clusters are
 * rescanned instead (same results). 0 forces rescanning. Set before prepare_workspace. */
int cora_set_vanguard_lows_budget(cora_engine *engine, uint64_t bytes);
/* Tuning knobs that never change results (the tests sweep them to cover every code path):
 *  "vanguard_lows_budget"  same as cora_set_vanguard_lows_budget;
 *  "warp_select_limit"     keys (0..256) one warp may collect while selecting the seeds of
 *                          a vanguard pair before it hands the pair to a block-wide
 *                          selection (0 sends every pair to the block selection);
 *  "topk_warp_limit"       the same for the threshold and final top-k of a query (k <= 32);
 *  "search_graphs"         1 (default): cora_search / cora_search_device replay a captured
 *                          CUDA graph of the whole search (rebuilt when the buffers, shape,
 *                          stream or configuration change; not used while profiling or
 *                          filter timing is on, nor on the legacy default stream); 0: every
 *                          search launches its kernels one by one. */
int cora_set_tuning(cora_engine *engine, const char *key, int64_t value);
/* 1 when the prepared workspace keeps vanguard lower bounds, 0 when it rescans, -1 on NULL. */
int cora_get_vanguard_mode(const cora_engine *engine);
/* Candidate capacity per query of the current workspace (array 7 above is nq x cap). */
uint64_t cora_get_candidate_capacity(const cora_engine *engine);

/* ---- Cluster-sharded search over several GPUs (no counterpart in the reference, which
 * searches on one GPU). One engine per GPU holds one shard: the clusters that
 * cora_shard_plan() gives its rank, with every centroid (each shard probes all of them).
 * A search runs on every shard with the same queries and arguments, in three calls with two
 * all-gathers in between, done by the caller (e.g. NCCL through torch.distributed) on the
 * same stream order:
 *   begin  (queries -> send)      all-gather send -> recv
 *   resume (recv -> send)         all-gather send -> recv
 *   end    (recv -> results)
 * send holds cora_shard_exchange_words(nq, k) u64; recv holds world of them, in rank order.
 * The first exchange carries each shard's k smallest vanguard seed distances (the global
 * pruning threshold is the k-th smallest of all), the second each shard's top-k (the result
 * is the top-k of all) plus its device error word, so that every rank reports a failure on
 * any shard. Results equal an unsharded search of the whole index, bit for bit. */

/* Loads a shard from arrays that hold only its own clusters (no counterpart in the
 * reference): for an index too large for one host, each rank builds or reads just the
 * clusters that cora_shard_plan(h_global_sizes, world) gives it. Arguments as
 * cora_load_from_raw_pointers, with the arrays in cluster order over the owned clusters
 * (local_vecs vectors), h_local_sizes[c] = h_global_sizes[c] for owned clusters and 0 for
 * the others (CORA_EINVAL otherwise), and every centroid. Call after cora_shard_configure;
 * with world 1 it loads the whole index. */
int cora_load_shard_arrays(cora_engine *engine, uint64_t local_vecs, uint64_t d, uint64_t p_d,
                           uint64_t n_centroids, uint64_t ex_b, const float *h_centroids,
                           const float *h_rotator, const uint32_t *h_short_data,
                           const float *h_short_factors, const uint8_t *h_long_code,
                           const float *h_ex_factors, const uint32_t *h_ids,
                           const uint64_t *h_local_sizes, const uint64_t *h_global_sizes);
/* Longest-processing-time plan over cluster sizes: owner_out[c] = shard of cluster c. */
int cora_shard_plan(const uint64_t *sizes, uint64_t nlist, uint32_t world, int32_t *owner_out);
/* Makes the engine load only shard `rank` of `world` (call before loading; world 1 = whole
 * index). CORA_ESTATE after a load. cora_search / cora_search_device are then rejected. */
int cora_shard_configure(cora_engine *engine, uint32_t rank, uint32_t world);
/* out[0..3] = rank, world, vectors held, clusters held. */
int cora_shard_info(const cora_engine *engine, uint64_t *out4);
uint64_t cora_shard_exchange_words(uint64_t num_queries, uint64_t topk);
/* Enqueue on `stream` (NULL: the engine's stream); return without synchronising. */
int cora_shard_search_begin(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                            uint64_t topk, uint64_t nprobe, uint64_t *d_send, void *stream);
/* Probing split by query over the shards (in place of cora_shard_search_begin): shard r
 * rotates every query but runs the probe GEMM and the exact top-nprobe only for queries
 * [r s, min(nq, (r + 1) s)), s = ceil(nq / world), writing that slice's probe lists to d_send
 * (cora_shard_probe_words(nq, nprobe, world) u64); after an all-gather of those buffers (rank
 * order), cora_shard_search_begin_probed takes every shard's slices and continues as
 * cora_shard_search_begin does (d_send: the first exchange's buffer). The probing stage then
 * costs each shard 1 / world of its single-GPU time; results are the same bits. */
uint64_t cora_shard_probe_words(uint64_t num_queries, uint64_t nprobe, uint32_t world);
int cora_shard_search_probe(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                            uint64_t topk, uint64_t nprobe, uint64_t *d_send, void *stream);
int cora_shard_search_begin_probed(cora_engine *engine, const uint64_t *d_recv, uint64_t *d_send);
int cora_shard_search_resume(cora_engine *engine, const uint64_t *d_recv, uint64_t *d_send);
int cora_shard_search_end(cora_engine *engine, const uint64_t *d_recv, float *d_final_dists,
                          uint32_t *d_final_pids);

/* Coarse probing that allocates nothing (no counterpart in the reference). For callers
 * that need a query's probe list where they cannot allocate device memory: e.g. a router
 * choosing the GPU or shard that owns a query's clusters while searches run beside it
 * (cudaMalloc/cudaFree would synchronise the device), or a process that cannot afford the
 * search workspace. Runs the search's own rotation, approximate-distance and guarded
 * top-nprobe kernels on `stream` (NULL: the engine's stream) and returns without
 * synchronising; needs a loaded index, not a workspace. Results equal what cora_search
 * probes for the same queries (cora_debug_copy arrays 1 and 2).
 *   d_queries      device, num_queries x dim f32
 *   d_probe_ids    device, num_queries x nprobe i32 (per query ascending by (distance, id))
 *   d_probe_dists  device, num_queries x nprobe f32 (exact squared distance to the centroid)
 * Intermediates live in one static device block of cora_probe_noalloc_scratch_limit()
 * bytes (16 MiB) per device; a call needing more is rejected with CORA_EINVAL (split the
 * queries). Nothing in the block needs to start at zero. The first call on each device
 * looks the block up (cudaGetSymbolAddress): make it before any stream capture (and again
 * the first call after the device's context was reset, which looks it up anew). The block
 * is shared by all engines of a device, so calls that overlap in time race on it:
 * serialise them (e.g. one stream). */
int cora_probe_noalloc(cora_engine *engine, const float *d_queries, uint64_t num_queries,
                       uint64_t nprobe, int32_t *d_probe_ids, float *d_probe_dists, void *stream);
uint64_t cora_probe_noalloc_scratch_limit(void);
/* Synchronises `stream` and reports a device-side failure of the last cora_probe_noalloc
 * on this device (a bounded wait in the tensor-core kernel that expired): CORA_ERUNTIME. */
int cora_probe_noalloc_status(cora_engine *engine, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* CORA_B200_H */
