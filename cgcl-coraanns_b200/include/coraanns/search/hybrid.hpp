// Header-only coraanns::HybridIndex over the C ABI of libcoraanns_b200.so.
//
// Same class name, method names, argument lists, defaults and exception types as the
// reference's include/coraanns/search/hybrid.cuh:18-203 and parameters.hpp:9-25, so code
// written against the reference (apps/search.cpp, the tests/gpu_*.cpp programs) compiles
// against this header instead; link with -lcoraanns_b200. Status codes map to exceptions:
// CORA_EINVAL -> std::invalid_argument, CORA_ESTATE -> std::logic_error, CORA_ENOMEM ->
// std::bad_alloc, anything else -> std::runtime_error (with the engine's message).
#pragma once

#include <climits>
#include <cstddef>
#include <cstdint>
#include <new>
#include <stdexcept>
#include <string>

#include "cora_b200.h"

namespace coraanns {

inline constexpr std::size_t default_vanguard_size = 5;
inline constexpr int default_batch_q = 4;
inline constexpr std::size_t max_query_chunk = 65535;
inline constexpr std::size_t max_probe_count = 65536;

inline void validate_search_shape(std::size_t queries, std::size_t topk, std::size_t nprobe,
                                  std::size_t centroids, std::size_t padded_dim) {
    if (queries == 0 || queries > max_query_chunk)
        throw std::invalid_argument("query count must be in [1, 65535]; split larger batches");
    if (topk == 0 || topk > INT_MAX / queries)
        throw std::invalid_argument("topk must be positive and queries * topk must fit an int");
    if (nprobe == 0 || nprobe > max_probe_count || nprobe > centroids)
        throw std::invalid_argument("nprobe must be in [1, min(nlist, 65536)]");
    if (centroids > INT_MAX / queries || padded_dim == 0 || padded_dim > INT_MAX / (queries * 4))
        throw std::invalid_argument("query workspace exceeds kernel indexing limits");
}

namespace queue {
using Position = std::uint64_t;
inline constexpr std::size_t default_capacity = std::size_t{1} << 26;
inline constexpr std::size_t default_spill_capacity = std::size_t{1} << 24;
}  // namespace queue

enum class KernelType { Lut4Bit, Bitwise };

namespace detail {
inline void check(int rc) {
    if (rc == CORA_OK) return;
    const std::string msg = cora_last_error();
    switch (rc) {
        case CORA_EINVAL: throw std::invalid_argument(msg);
        case CORA_ESTATE: throw std::logic_error(msg);
        case CORA_ENOMEM: throw std::bad_alloc();
        default: throw std::runtime_error(msg);
    }
}
}  // namespace detail

class HybridIndex {
  public:
    explicit HybridIndex(int device = 0) { detail::check(cora_create(&engine_, device)); }
    HybridIndex(const HybridIndex &) = delete;
    HybridIndex &operator=(const HybridIndex &) = delete;
    ~HybridIndex() { cora_destroy(engine_); }

    void set_profiling(bool enabled) { cora_set_profiling(engine_, enabled); }
    void set_candidate_stats(bool enabled) { cora_set_candidate_stats(engine_, enabled); }
    void set_gpu_filter_timing(bool enabled) { cora_set_gpu_filter_timing(engine_, enabled); }
    void set_cross_query_reuse(bool enabled) { cora_set_cross_query_reuse(engine_, enabled); }
    void set_cpu_secondary_filter(bool enabled) { cora_set_cpu_secondary_filter(engine_, enabled); }

    queue::Position get_last_submitted_count() const { return cora_get_last_submitted_count(engine_); }
    queue::Position get_last_spilled_count() const { return cora_get_last_spilled_count(engine_); }
    void set_queue_capacity(std::size_t capacity) {
        detail::check(cora_set_queue_capacity(engine_, capacity));
    }
    void set_queue_spill_capacity(std::size_t capacity) {
        detail::check(cora_set_queue_spill_capacity(engine_, capacity));
    }
    std::size_t get_queue_capacity() const { return cora_get_queue_capacity(engine_); }
    std::size_t get_last_refined_count() const { return cora_get_last_refined_count(engine_); }
    float get_last_gpu_filter_ms() const { return cora_get_last_gpu_filter_ms(engine_); }

    void set_vanguard_size(std::size_t size) { detail::check(cora_set_vanguard_size(engine_, size)); }
    std::size_t get_vanguard_size() const { return cora_get_vanguard_size(engine_); }

    void set_ip_kernel_type(KernelType t) { cora_set_ip_kernel_type(engine_, static_cast<int>(t)); }
    KernelType get_ip_kernel_type() const {
        return static_cast<KernelType>(cora_get_ip_kernel_type(engine_));
    }
    // Distance (this engine's addition; the reference's hybrid path is L2 only): 0 squared
    // L2, 1 inner product. Set from the file header by load_index_file.
    void set_metric(int metric) { detail::check(cora_set_metric(engine_, metric)); }
    int get_metric() const { return cora_get_metric(engine_); }
    // Refinement form (this engine's addition): false = the reference's 128 ip1 + ip2.
    void set_refine_full_code(bool enabled) { cora_set_refine_full_code(engine_, enabled ? 1 : 0); }
    bool get_refine_full_code() const { return cora_get_refine_full_code(engine_) != 0; }

    void prepare_workspace(std::size_t max_queries, std::size_t max_topk, std::size_t max_nprobe) {
        detail::check(cora_prepare_workspace(engine_, max_queries, max_topk, max_nprobe));
    }
    void free_workspace() noexcept { cora_free_workspace(engine_); }
    void reset_buffer(const float *h_queries, std::size_t num_queries) {
        detail::check(cora_reset_buffer(engine_, h_queries, num_queries));
    }

    // The diagnostic FP32 refinement against a mapped base (hybrid.cuh:171-178): candidates
    // are ranked by their exact squared L2 distance to base row `original id`; the rows the
    // engine holds are copied into HBM by this call (or when the index is loaded).
    void enable_exact_refine(const std::uint8_t *base_mapping, std::size_t base_rows,
                             std::size_t base_dim, std::size_t row_stride_bytes,
                             std::size_t data_offset_bytes) {
        detail::check(cora_enable_exact_refine(engine_, base_mapping, base_rows, base_dim,
                                               row_stride_bytes, data_offset_bytes));
    }

    // Unlike the reference, the extended codes, factors and ids are copied to HBM: the host
    // arrays need to live only for the duration of the call.
    void load_from_raw_pointers(std::size_t num_vecs, std::size_t d, std::size_t p_d,
                                std::size_t n_centroids, std::size_t ex_b,
                                const float *h_centroids, const float *h_rotator,
                                const std::uint32_t *h_short_data, const float *h_short_factors,
                                const std::uint8_t *h_long_code, const float *h_ex_factors,
                                const std::uint32_t *h_ids, const std::size_t *h_cluster_sizes) {
        static_assert(sizeof(std::size_t) == sizeof(std::uint64_t), "LP64 expected");
        detail::check(cora_load_from_raw_pointers(
            engine_, num_vecs, d, p_d, n_centroids, ex_b, h_centroids, h_rotator, h_short_data,
            h_short_factors, h_long_code, h_ex_factors, h_ids,
            reinterpret_cast<const std::uint64_t *>(h_cluster_sizes)));
    }
    // IVF::load + index::SearchData + load_from_raw_pointers in one step.
    void load_index_file(const std::string &path) {
        detail::check(cora_load_index_file(engine_, path.c_str()));
    }

    void capture_thresholds(float *out, std::size_t nq) const {
        detail::check(cora_capture_thresholds(engine_, out, nq));
    }
    void seed_thresholds(const float *in, std::size_t nq) {
        detail::check(cora_seed_thresholds(engine_, in, nq));
    }

    void search(const float *h_queries, std::size_t num_queries, std::size_t topk,
                std::size_t nprobe, float *h_final_dists, std::uint32_t *h_final_pids,
                int batch_q = default_batch_q) {
        detail::check(cora_search(engine_, h_queries, num_queries, topk, nprobe, h_final_dists,
                                  h_final_pids, batch_q));
    }

    // Shape of the loaded index (no reference counterpart: the reference reads it from IVF).
    struct Shape {
        std::size_t num_vectors, dim, padded_dim, num_clusters, ex_bits, max_cluster_size;
    };
    Shape index_info() const {
        std::uint64_t v[6];
        detail::check(cora_index_info(engine_, v));
        return Shape{v[0], v[1], v[2], v[3], v[4], v[5]};
    }

    cora_engine *handle() { return engine_; }

  private:
    cora_engine *engine_ = nullptr;
};

}  // namespace coraanns
