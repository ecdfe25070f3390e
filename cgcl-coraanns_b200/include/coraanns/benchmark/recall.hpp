// recall@k for the coraanns_search CLI, with the reference evaluator's semantics
// (include/coraanns/benchmark/recall.hpp:52-275): a returned id counts once; it is a hit if it
// is among the ground-truth top-k ids, or (distance-aware mode, with a base file) if its exact
// fp64 score is as good as the ground truth's rank-k neighbour's: squared L2 distance <= it
// (metric 0), or inner product >= it (metric 1). Ids that are out of range or equal to
// UINT32_MAX are misses.
#pragma once

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <iostream>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "coraanns/benchmark/vectors.hpp"

namespace coraanns::bench {

struct RecallCounts {
    std::size_t total = 0, id_hits = 0, distance_hits = 0, exact_checks = 0;
    std::size_t correct() const { return id_hits + distance_hits; }
};

class RecallEvaluator {
  public:
    RecallEvaluator(const float *queries, std::size_t nq, std::size_t dim,
                    const Matrix<uint32_t> &gt, std::size_t topk, const std::string &base_file,
                    int metric = 0)
        : queries_(queries), nq_(nq), dim_(dim), topk_(topk), metric_(metric) {
        if (!queries || !nq || !dim || !topk || gt.rows != nq || gt.cols < topk)
            throw std::invalid_argument("Invalid query/GT shape for recall@k");
        if (metric != 0 && metric != 1) throw std::invalid_argument("Recall metric must be L2 or IP");
        if (!base_file.empty()) {
            base_ = std::make_unique<MappedVectors>(base_file);
            if (base_->dim() != dim) throw std::invalid_argument("Recall base and query dimensions differ");
        }
        truth_.resize(nq * topk);
        radius_.assign(nq, 0.0);
        for (std::size_t q = 0; q < nq; ++q) {
            uint32_t *t = truth_.data() + q * topk;
            for (std::size_t j = 0; j < topk; ++j) {
                t[j] = gt(q, j);
                if (t[j] == UINT32_MAX || (base_ && t[j] >= base_->rows()))
                    throw std::invalid_argument("Invalid GT ID for recall base");
            }
            if (base_) {
                radius_[q] = score(q, t[topk - 1]);
                if (!finite(radius_[q])) throw std::invalid_argument("Non-finite query/GT distance");
            }
            std::sort(t, t + topk);
            if (std::adjacent_find(t, t + topk) != t + topk)
                throw std::invalid_argument("GT top-k contains duplicate IDs");
        }
        std::cout << "[Recall] mode=" << (base_ ? "distance-aware" : "id")
                  << " metric=" << (metric_ == 0 ? "l2" : "ip") << " topk=" << topk
                  << " base=" << (base_ ? base_file : "none (use --recall-base for distance checks)")
                  << "\n";
    }

    RecallCounts count_query(std::size_t q, const uint32_t *res, std::size_t count) const {
        RecallCounts c;
        c.total = topk_;
        std::vector<uint32_t> ids;
        for (std::size_t j = 0; j < std::min(count, topk_); ++j)
            if (res[j] != UINT32_MAX && (!base_ || res[j] < base_->rows())) ids.push_back(res[j]);
        std::sort(ids.begin(), ids.end());
        ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
        const uint32_t *t = truth_.data() + q * topk_;
        for (uint32_t id : ids) {
            if (std::binary_search(t, t + topk_, id)) {
                ++c.id_hits;
            } else if (base_) {
                const double s = score(q, id);
                ++c.exact_checks;
                c.distance_hits += finite(s) && (metric_ == 0 ? s <= radius_[q] : s >= radius_[q]);
            }
        }
        return c;
    }

    double evaluate(const std::vector<uint32_t> &results) const {
        if (results.size() < nq_ * topk_) throw std::invalid_argument("Result array is smaller than nq * topk");
        const auto t0 = std::chrono::steady_clock::now();
        std::vector<RecallCounts> per(nq_);
#pragma omp parallel for schedule(static) if (base_ && nq_ >= 128)
        for (std::size_t q = 0; q < nq_; ++q) per[q] = count_query(q, results.data() + q * topk_, topk_);
        RecallCounts c;
        for (const auto &p : per) {
            c.total += p.total;
            c.id_hits += p.id_hits;
            c.distance_hits += p.distance_hits;
            c.exact_checks += p.exact_checks;
        }
        const double ms =
            std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        const double denom = static_cast<double>(c.total);
        const double recall = c.correct() / denom;
        std::cout << "[RecallEval] id_recall=" << c.id_hits / denom << " recall=" << recall
                  << " distance_hits=" << c.distance_hits << " exact_checks=" << c.exact_checks
                  << " eval_ms=" << ms << '\n';
        return recall;
    }

  private:
    static bool finite(double v) {
        uint64_t b;
        std::memcpy(&b, &v, 8);
        return (b & 0x7ff0000000000000ULL) != 0x7ff0000000000000ULL;
    }
    // exact fp64 score: squared L2 distance (metric 0) or inner product (metric 1)
    double score(std::size_t q, uint32_t id) const {
        const float *a = queries_ + q * dim_;
        const float *b = base_->row(id);
        double s = 0.0;
        for (std::size_t d = 0; d < dim_; ++d) {
            if (metric_ == 0) {
                const double e = static_cast<double>(a[d]) - b[d];
                s += e * e;
            } else {
                s += static_cast<double>(a[d]) * b[d];
            }
        }
        return s;
    }

    const float *queries_;
    std::size_t nq_, dim_, topk_;
    int metric_ = 0;
    std::unique_ptr<MappedVectors> base_;
    std::vector<uint32_t> truth_;
    std::vector<double> radius_;
};

}  // namespace coraanns::bench
