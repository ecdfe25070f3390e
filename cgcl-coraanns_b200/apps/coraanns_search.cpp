// coraanns_search: the batch search benchmark with the reference CLI's arguments and report
// lines (apps/search.cpp:26-318), running the B200 engine through coraanns::HybridIndex.
//
//   coraanns_search <index_file> <query_file> <gt_file> [--topk 100] [--nprobes 40,50,...]
//       [--rounds 5] [--warmup 1] [--batch-q 4] [--query-chunk N] [--threads N]
//       [--vanguard-size 5] [--cpu-secondary-filter true] [--queue-capacity 67108864]
//       [--queue-spill-capacity 16777216] [--cross-query-reuse true] [--candidate-stats false]
//       [--gpu-filter-timing false] [--profile false] [--exact-base FILE]
//       [--recall-base FILE] [--recall-once false]
//
// The index file is loaded straight into HBM by the engine (IVF::load + SearchData in one
// native step). QPS counts every query of every chunk, host copies included, like the
// reference's stopwatch around reset_buffer + search.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <iostream>
#include <limits>
#include <memory>
#include <string>
#include <vector>

#include <omp.h>

#include "coraanns/benchmark/options.hpp"
#include "coraanns/benchmark/recall.hpp"
#include "coraanns/benchmark/vectors.hpp"
#include "coraanns/search/hybrid.hpp"

namespace {

void print_usage(const char *program) {
    std::cerr << "Usage: " << program
              << " <index_file> <query_file> <gt_file>"
                 " [--topk 100] [--nprobes 40,50,...] [--rounds 5]"
                 " [--warmup 1] [--batch-q 4] [--query-chunk N] [--threads N]"
                 " [--vanguard-size 5] [--cpu-secondary-filter true]"
                 " [--queue-capacity 67108864] [--queue-spill-capacity 16777216]"
                 " [--cross-query-reuse true] [--candidate-stats false]"
                 " [--gpu-filter-timing false] [--profile false]"
                 " [--exact-base FILE] [--recall-base FILE] [--recall-once false]\n";
}

struct ChunkStats {
    unsigned long long submitted = 0, refined = 0, spilled = 0, wraps = 0;
    double gpu_filter_ms = 0.0;
};

}  // namespace

int main(int argc, char **argv) {
    if (argc < 4) {
        print_usage(argv[0]);
        return 1;
    }
    using namespace coraanns::bench;
    try {
        const std::string recall_base = take_recall_base(argc, argv);
        const std::string index_file = argv[1], query_file = argv[2], gt_file = argv[3];
        // the reference CLI's options (apps/search.cpp:26-318), in the order they are read
        OptionTable opt{{"topk", OptionKind::kSize},
                        {"rounds", OptionKind::kSize},
                        {"warmup", OptionKind::kSize},
                        {"recall-once", OptionKind::kBool},
                        {"batch-q", OptionKind::kSize},
                        {"threads", OptionKind::kSize},
                        {"vanguard-size", OptionKind::kSize},
                        {"profile", OptionKind::kBool},
                        {"candidate-stats", OptionKind::kBool},
                        {"gpu-filter-timing", OptionKind::kBool},
                        {"cross-query-reuse", OptionKind::kBool},
                        {"cpu-secondary-filter", OptionKind::kBool},
                        {"queue-capacity", OptionKind::kSize},
                        {"queue-spill-capacity", OptionKind::kSize},
                        {"query-chunk", OptionKind::kSize},
                        {"exact-base", OptionKind::kText},
                        {"nprobes", OptionKind::kText}};
        opt.parse(argc, argv, 4);
        const std::size_t topk = opt.size("topk", 100);
        const std::size_t rounds = opt.size("rounds", 5);
        const std::size_t warmup = opt.size("warmup", 1);
        const bool recall_once = opt.flag("recall-once", false);
        const std::size_t batch_q = opt.size("batch-q", coraanns::default_batch_q);
        if (batch_q < 1 || batch_q > 6) throw std::invalid_argument("batch-q must be in [1, 6]");
        const std::size_t threads = opt.size("threads", static_cast<std::size_t>(omp_get_max_threads()));
        if (threads == 0 || threads > static_cast<std::size_t>(std::numeric_limits<int>::max()))
            throw std::invalid_argument("threads must be a positive int");
        omp_set_dynamic(0);
        omp_set_num_threads(static_cast<int>(threads));
        const std::size_t vanguard = opt.size("vanguard-size", coraanns::default_vanguard_size);
        const bool profile = opt.flag("profile", false);
        const bool candidate_stats = opt.flag("candidate-stats", false);
        const bool filter_timing = opt.flag("gpu-filter-timing", false);
        const bool reuse = opt.flag("cross-query-reuse", true);
        const bool secondary = opt.flag("cpu-secondary-filter", true);
        const std::size_t qcap = opt.size("queue-capacity", coraanns::queue::default_capacity);
        const std::size_t scap = opt.size("queue-spill-capacity", coraanns::queue::default_spill_capacity);
        if (qcap == 0 || (qcap & (qcap - 1)) != 0)
            throw std::invalid_argument("queue-capacity must be a positive power of two");

        std::cout << "Loading queries and groundtruth..." << std::endl;
        const Matrix<float> query = load_vectors<float>(query_file);
        const Matrix<uint32_t> gt = load_vectors<uint32_t>(gt_file);
        const std::size_t nq = query.rows, dim = query.cols;
        std::cout << "Loaded " << nq << " queries with dimension " << dim << std::endl;
        const std::size_t chunk_req = opt.size("query-chunk", nq);
        if (chunk_req == 0) throw std::invalid_argument("query-chunk must be positive");
        const std::size_t chunk = std::min({chunk_req, nq, coraanns::max_query_chunk});

        std::cout << "Initializing GPU Index..." << std::endl;
        coraanns::HybridIndex index;
        index.load_index_file(index_file);
        const auto shape = index.index_info();
        // --exact-base: FP32 diagnostic refine against a mapped base (apps/search.cpp:126-146,
        // 171-175); exact distances are squared L2, the metric of the hybrid search path
        std::unique_ptr<MappedVectors> exact_base;
        const std::string exact_base_file = opt.text("exact-base", "");
        if (!exact_base_file.empty()) {
            exact_base = std::make_unique<MappedVectors>(exact_base_file);
            if (exact_base->rows() != shape.num_vectors || exact_base->dim() != shape.dim) {
                std::cerr << "Exact-refine base shape mismatch: file=" << exact_base->rows() << 'x'
                          << exact_base->dim() << ", index=" << shape.num_vectors << 'x'
                          << shape.dim << '\n';
                return 1;
            }
            std::cout << "Exact FP32 refine enabled with mmap base: " << exact_base_file << " ("
                      << exact_base->rows() << 'x' << exact_base->dim() << ")\n";
            index.enable_exact_refine(exact_base->mapping(), exact_base->rows(), exact_base->dim(),
                                      exact_base->row_stride_bytes(),
                                      exact_base->data_offset_bytes());
        }
        std::unique_ptr<RecallEvaluator> evaluator;
        if (!recall_once)
            evaluator = std::make_unique<RecallEvaluator>(query.data.data(), nq, dim, gt, topk,
                                                          recall_base, index.get_metric());
        validate_benchmark_shape(nq, dim, gt.rows, gt.cols, shape.dim, topk, rounds);
        const auto nprobes = parse_nprobes(opt.text("nprobes", ""), shape.num_clusters);
        const std::size_t max_nprobe = *std::max_element(nprobes.begin(), nprobes.end());
        coraanns::validate_search_shape(chunk, topk, max_nprobe, shape.num_clusters, shape.padded_dim);

        index.set_profiling(profile);
        index.set_candidate_stats(candidate_stats);
        index.set_gpu_filter_timing(filter_timing);
        index.set_cross_query_reuse(reuse);
        index.set_cpu_secondary_filter(secondary);
        index.set_vanguard_size(vanguard);
        std::cout << "Max cluster size: " << shape.max_cluster_size << std::endl;
        index.set_queue_capacity(qcap);
        index.set_queue_spill_capacity(scap);
        std::cout << "Allocating GPU workspace...\n";
        index.prepare_workspace(chunk, topk, max_nprobe);

        std::cout << "Algorithm: CoraANN (B200 scan + on-GPU refinement)\n"
                  << "topk: " << topk << "\nbatch_q: " << batch_q << "\nquery_chunk: " << chunk
                  << "\ncpu_threads: " << threads << "\nqueue_capacity: " << qcap
                  << "\nqueue_spill_capacity: " << scap << "\nvanguard_size: " << vanguard
                  << "\ncpu_secondary_filter: " << (secondary ? "true" : "false")
                  << "\ncross_query_reuse: " << (reuse ? "true" : "false")
                  << "\ncandidate_stats: " << (candidate_stats ? "true" : "false")
                  << "\ngpu_filter_timing: " << (filter_timing ? "true" : "false")
                  << "\nrounds: " << rounds << "\nwarmup_rounds: " << warmup
                  << "\nprofile: " << (profile ? "true" : "false") << "\nnprobes: " << join_values(nprobes)
                  << '\n';

        const std::size_t L = nprobes.size();
        std::vector<std::vector<double>> qps(rounds, std::vector<double>(L));
        std::vector<std::vector<double>> recall(recall_once ? 1 : rounds, std::vector<double>(L));
        std::vector<std::vector<uint32_t>> saved(recall_once ? L : 0, std::vector<uint32_t>(nq * topk));
        if (recall_once)
            std::cout << "[RecallSchedule] policy=once-after-benchmark source_round=1 evaluations=" << L << '\n';
        std::vector<float> dists(nq * topk);
        std::vector<uint32_t> ids(nq * topk);

        auto run_all = [&](std::size_t nprobe) {
            ChunkStats s;
            for (std::size_t b = 0; b < nq; b += chunk) {
                const std::size_t n = std::min(chunk, nq - b);
                const float *q = query.row(b);
                index.reset_buffer(q, n);
                index.search(q, n, topk, nprobe, dists.data() + b * topk, ids.data() + b * topk,
                             static_cast<int>(batch_q));
                const auto sub = index.get_last_submitted_count();
                s.submitted += sub;
                s.refined += index.get_last_refined_count();
                s.spilled += index.get_last_spilled_count();
                s.gpu_filter_ms += index.get_last_gpu_filter_ms();
                s.wraps += sub == 0 ? 0 : (sub - 1) / qcap;
            }
            return s;
        };

        std::cout << "Starting batch benchmark..." << std::endl;
        for (std::size_t l = 0; l < L; ++l) {
            const std::size_t nprobe = nprobes[l];
            for (std::size_t w = 0; w < warmup; ++w) run_all(nprobe);
            for (std::size_t r = 0; r < rounds; ++r) {
                const auto t0 = std::chrono::steady_clock::now();
                const ChunkStats s = run_all(nprobe);
                const double us =
                    std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
                qps[r][l] = static_cast<double>(nq) / (us / 1e6);
                if (recall_once) {
                    if (r == 0) saved[l] = ids;
                } else {
                    recall[r][l] = evaluator->evaluate(ids);
                }
                std::cout << "[Run] round=" << (r + 1) << " nprobe=" << nprobe << " QPS=" << qps[r][l];
                if (recall_once)
                    std::cout << " recall=deferred\n";
                else
                    std::cout << " recall=" << recall[r][l] << '\n';
                std::printf("[QueueStats] round=%zu nprobe=%zu submitted=%llu spilled=%llu wraps=%llu\n",
                            r + 1, nprobe, s.submitted, s.spilled, s.wraps);
                if (candidate_stats)
                    std::printf("[CandidateStats] round=%zu nprobe=%zu queries=%zu submitted=%llu "
                                "actual_refined=%llu submitted_per_query=%.6f actual_refined_per_query=%.6f\n",
                                r + 1, nprobe, nq, s.submitted, s.refined,
                                static_cast<double>(s.submitted) / nq, static_cast<double>(s.refined) / nq);
                if (filter_timing)
                    std::printf("[GPUFilter] round=%zu nprobe=%zu queries=%zu total_ms=%.6f ms_per_query=%.9f\n",
                                r + 1, nprobe, nq, s.gpu_filter_ms, s.gpu_filter_ms / nq);
                std::fflush(stdout);
            }
        }
        if (recall_once) {
            std::cout << "[RecallSchedule] QPS rounds complete; evaluating saved results" << std::endl;
            evaluator = std::make_unique<RecallEvaluator>(query.data.data(), nq, dim, gt, topk,
                                                          recall_base, index.get_metric());
            for (std::size_t l = 0; l < L; ++l) {
                recall[0][l] = evaluator->evaluate(saved[l]);
                std::cout << "[RecallPoint] nprobe=" << nprobes[l] << " source_round=1 recall=" << recall[0][l]
                          << '\n';
            }
        }
        std::cout << "nprobe\tQPS\trecall\n";
        for (std::size_t l = 0; l < L; ++l) {
            double q = 0, rc = 0;
            for (std::size_t r = 0; r < rounds; ++r) q += qps[r][l];
            for (const auto &row : recall) rc += row[l];
            std::cout << nprobes[l] << '\t' << q / rounds << '\t' << rc / recall.size() << '\n';
        }
    } catch (const std::exception &e) {
        std::cerr << "coraanns_search failed: " << e.what() << '\n';
        print_usage(argv[0]);
        return 1;
    }
    return 0;
}
