// Test infrastructure only: a thin C-ABI harness over the reference's OWN CPU code,
// compiled from the read-only reference tree by oracle/Makefile into oracle/_ref/.
// Nothing in the product links or loads this; tests, smoke() and bench.py's CPU
// baseline / reference arm use it as the checker and as the timed host-CPU path.
//
// What each entry point runs (paths are within the reference project):
//   ref_build_index   rabitqlib::ivf::IVF(n, dim, k, bits, metric).construct() + save()
//                     third_party/rabitq/include/rabitqlib/index/ivf/ivf.hpp:221-303,403-445
//   ref_open/ref_info IVF::load()                                   ivf.hpp:447-539
//   ref_search_data   coraanns::index::SearchData (file layout -> packed GPU arrays)
//                     src/index/search_data.cpp:9-127
//   ref_search        IVF::search() over queries with OpenMP, exactly as the rabitq_cpu
//                     baseline does (apps/baselines/cpu.cpp:110-115)
//   ref_ip_ex         select_excode_ipfunc(ex_bits) (utils/space.hpp:777-805), i.e.
//                     ip64_fxu7_avx for 7 ex bits (utils/space.hpp:677-762)
//   ref_pack_ex7      packing_7bit_excode (quantization/pack_excode.hpp:216-264)
//   ref_recall        recall_eval::Evaluator (include/coraanns/benchmark/recall.hpp:74-275)
#include <omp.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

#include "coraanns/benchmark/recall.hpp"
#include "coraanns/index/search_data.hpp"
#include "rabitqlib/defines.hpp"
#include "rabitqlib/index/ivf/ivf.hpp"
#include "rabitqlib/quantization/pack_excode.hpp"
#include "rabitqlib/utils/space.hpp"

namespace {
thread_local std::string g_error;

int fail(const std::exception &e) {
    g_error = e.what();
    return -1;
}

struct Handle {
    rabitqlib::ivf::IVF ivf;
};

struct IdMatrixView {
    const uint32_t *data;
    long r, c;
    long rows() const { return r; }
    long cols() const { return c; }
    uint32_t operator()(long i, long j) const { return data[i * c + j]; }
};
}  // namespace

extern "C" {

const char *ref_last_error() { return g_error.c_str(); }

int ref_build_index(const float *data, uint64_t n, uint64_t dim, const float *centroids,
                    uint64_t k, const uint32_t *cluster_ids, int total_bits, int metric_ip,
                    int faster, const char *path) {
    try {
        rabitqlib::ivf::IVF ivf(n, dim, k, total_bits,
                                metric_ip ? rabitqlib::METRIC_IP : rabitqlib::METRIC_L2);
        ivf.construct(data, centroids, cluster_ids, faster != 0);
        ivf.save(path);
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

void *ref_open(const char *path) {
    try {
        auto h = std::make_unique<Handle>();
        h->ivf.load(path);
        return h.release();
    } catch (const std::exception &e) {
        fail(e);
        return nullptr;
    }
}

void ref_close(void *handle) { delete static_cast<Handle *>(handle); }

// out: num, dim, padded_dim, nlist, ex_bits, metric
int ref_info(void *handle, uint64_t *out) {
    auto &ivf = static_cast<Handle *>(handle)->ivf;
    out[0] = ivf.num_vectors();
    out[1] = ivf.dim();
    out[2] = ivf.padded_dim();
    out[3] = ivf.num_clusters();
    out[4] = ivf.ex_bits();
    out[5] = static_cast<uint64_t>(ivf.metric_type());
    return 0;
}

int ref_ids(void *handle, uint32_t *out) {
    auto &ivf = static_cast<Handle *>(handle)->ivf;
    std::memcpy(out, ivf.ids(), ivf.num_vectors() * sizeof(uint32_t));
    return 0;
}

// Runs the reference adapter on a freshly loaded copy of the index (the adapter takes
// ownership of the extended codes) and copies every packed array into caller buffers.
int ref_search_data(const char *path, float *centroids, float *rotator, uint32_t *short_data,
                    float *short_factors, uint8_t *long_codes, float *ex_factors,
                    uint64_t *cluster_sizes) {
    try {
        rabitqlib::ivf::IVF ivf;
        ivf.load(path);
        coraanns::index::SearchData sd(ivf, true, 1);
        const size_t n = ivf.num_vectors(), D = ivf.padded_dim();
        const size_t lc = (D * ivf.ex_bits() + 7) / 8;
        std::memcpy(centroids, sd.h_centroids.data(), sd.h_centroids.size() * sizeof(float));
        std::memcpy(rotator, sd.host_rotator.data(), sd.host_rotator.size() * sizeof(float));
        std::memcpy(short_data, sd.host_short_data.data(),
                    sd.host_short_data.size() * sizeof(uint32_t));
        std::memcpy(short_factors, sd.host_short_factors.data(),
                    sd.host_short_factors.size() * sizeof(float));
        std::memcpy(long_codes, sd.host_long_codes, n * lc);
        std::memcpy(ex_factors, sd.host_ex_factors.data(),
                    sd.host_ex_factors.size() * sizeof(float));
        for (size_t c = 0; c < sd.cluster_sizes.size(); ++c)
            cluster_sizes[c] = sd.cluster_sizes[c];
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

int ref_search(void *handle, const float *queries, uint64_t nq, uint64_t k, uint64_t nprobe,
               uint32_t *out, int threads, int hacc) {
    try {
        auto &ivf = static_cast<Handle *>(handle)->ivf;
        const size_t dim = ivf.dim();
        omp_set_dynamic(0);
#pragma omp parallel for schedule(static) num_threads(threads)
        for (int64_t i = 0; i < static_cast<int64_t>(nq); ++i) {
            ivf.search(queries + i * dim, k, nprobe, out + i * k, hacc != 0);
        }
        return 0;
    } catch (const std::exception &e) {
        return fail(e);
    }
}

float ref_ip_ex(const float *query, const uint8_t *code, uint64_t padded_dim, uint64_t ex_bits) {
    return rabitqlib::select_excode_ipfunc(ex_bits)(query, code, padded_dim);
}

void ref_pack_ex7(const uint8_t *raw, uint8_t *compact, uint64_t padded_dim) {
    rabitqlib::quant::rabitq_impl::ex_bits::packing_7bit_excode(raw, compact, padded_dim);
}

double ref_recall(const float *queries, uint64_t nq, uint64_t dim, const uint32_t *gt,
                  uint64_t gt_cols, uint64_t topk, const char *base_file, int metric_ip,
                  const uint32_t *results) {
    try {
        IdMatrixView view{gt, static_cast<long>(nq), static_cast<long>(gt_cols)};
        recall_eval::Evaluator ev(queries, nq, dim, view, topk, base_file ? base_file : "",
                                  metric_ip ? rabitqlib::METRIC_IP : rabitqlib::METRIC_L2);
        std::vector<uint32_t> r(results, results + nq * topk);
        return ev.evaluate(r);
    } catch (const std::exception &e) {
        fail(e);
        return -1.0;
    }
}

}  // extern "C"
