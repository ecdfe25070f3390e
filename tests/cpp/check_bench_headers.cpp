// Unit checks of the CLI's option parser, vector-file readers and recall evaluator
// (host code only; no GPU). Built and run by tests/test_cli.py. Exits non-zero on failure.
#include <cstdio>
#include <fstream>
#include <functional>
#include <string>
#include <vector>

#include "coraanns/benchmark/options.hpp"
#include "coraanns/benchmark/recall.hpp"
#include "coraanns/benchmark/vectors.hpp"

using namespace coraanns::bench;

static int failures = 0;
#define CHECK(c)                                                      \
    do {                                                              \
        if (!(c)) {                                                   \
            std::fprintf(stderr, "FAIL %s:%d %s\n", __FILE__, __LINE__, #c); \
            ++failures;                                               \
        }                                                             \
    } while (0)

static bool throws(const std::function<void()> &f) {
    try {
        f();
    } catch (const std::exception &) {
        return true;
    }
    return false;
}

static OptionTable parse(std::vector<std::string> args) {
    std::vector<char *> argv;
    for (auto &a : args) argv.push_back(a.data());
    argv.push_back(nullptr);
    OptionTable t{{"topk", OptionKind::kSize},
                  {"rounds", OptionKind::kSize},
                  {"nprobes", OptionKind::kText},
                  {"profile", OptionKind::kBool},
                  {"absent", OptionKind::kBool}};
    t.parse(static_cast<int>(args.size()), argv.data(), 0);
    return t;
}

static std::string message_of(const std::function<void()> &f) {
    try {
        f();
    } catch (const std::exception &e) {
        return e.what();
    }
    return "";
}

int main(int argc, char **argv) {
    const std::string dir = argc > 1 ? argv[1] : ".";
    // options: the reference's syntax and messages
    auto o = parse({"--topk", "10", "--nprobes=4,8", "--profile", "on"});
    CHECK(o.size("topk", 0) == 10);
    CHECK(o.size("rounds", 5) == 5);
    CHECK(o.text("nprobes", "") == "4,8");
    CHECK(o.flag("profile", false));
    CHECK(!o.flag("absent", false));
    CHECK(o.given("topk") && !o.given("rounds"));
    CHECK(parse({"--topk="}).size("topk", 7) == 7);  // empty value: not given
    CHECK(message_of([] { parse({"--bogus", "1"}); }) == "Unknown option --bogus");
    CHECK(message_of([] { parse({"--topk", "1", "--topk", "2"}); }) ==
          "Invalid or duplicate option --topk");
    CHECK(message_of([] { parse({"--topk"}); }) == "Missing value for --topk");
    CHECK(message_of([] { parse({"--topk", "--rounds", "2"}); }) == "Missing value for --topk");
    CHECK(message_of([] { parse({"positional"}); }) == "Unexpected positional argument: positional");
    CHECK(message_of([] { parse({"--topk", "-1"}); }) == "Invalid integer for --topk: -1");
    CHECK(message_of([] { parse({"--topk", "12x"}); }) == "Invalid integer for --topk: 12x");
    CHECK(message_of([] { parse({"--topk", "99999999999999999999999"}); }) ==
          "Invalid integer for --topk: 99999999999999999999999");
    CHECK(message_of([] { parse({"--profile", "maybe"}); }) == "Invalid boolean for --profile: maybe");
    CHECK(!parse({"--profile=off"}).flag("profile", true));
    CHECK(throws([] { parse({}).size("profile", 0); }));   // read as the wrong kind
    CHECK(throws([] { parse({}).flag("undeclared", 0); }));
    CHECK(parse_nprobes("4,8", 16) == (std::vector<std::size_t>{4, 8}));
    CHECK(parse_nprobes("", 16) == (std::vector<std::size_t>{16}));
    CHECK(parse_nprobes("", 100) == (std::vector<std::size_t>{40, 50, 60, 75, 95}));
    CHECK(throws([] { parse_nprobes("0", 16); }));
    CHECK(throws([] { parse_nprobes("17", 16); }));
    CHECK(throws([] { parse_nprobes("4,4", 16); }));
    CHECK(throws([] { parse_nprobes("4,,8", 16); }));
    CHECK(throws([] { parse_nprobes("+4", 16); }));
    CHECK(throws([] { parse_nprobes("4,", 16); }));
    CHECK(message_of([] { parse_nprobes("4,4", 16); }) == "Duplicate nprobe value: 4");
    CHECK(message_of([] { parse_nprobes("17", 16); }) == "Each nprobe must be in [1, nlist]; got: 17");
    CHECK(join_values({4, 8, 16}) == "4,8,16");
    CHECK(throws([] { validate_benchmark_shape(10, 8, 9, 10, 8, 10, 1); }));
    CHECK(throws([] { validate_benchmark_shape(10, 8, 10, 5, 8, 10, 1); }));
    CHECK(throws([] { validate_benchmark_shape(10, 8, 10, 10, 9, 10, 1); }));
    CHECK(!throws([] { validate_benchmark_shape(10, 8, 10, 10, 8, 10, 1); }));
    {
        std::vector<std::string> a = {"prog", "i", "--recall-base=base.fbin", "q", "g", "--topk", "3"};
        std::vector<char *> v;
        for (auto &s : a) v.push_back(s.data());
        v.push_back(nullptr);
        int n = static_cast<int>(a.size());
        CHECK(take_recall_base(n, v.data()) == "base.fbin");
        CHECK(n == 6 && std::string(v[3]) == "g" && v[6] == nullptr);
    }

    // vector files: 3 rows x 2 dims, .fvecs and .fbin
    const float rows[3][2] = {{0.f, 0.f}, {1.f, 0.f}, {0.f, 3.f}};
    {
        std::ofstream f(dir + "/b.fvecs", std::ios::binary);
        for (auto &r : rows) {
            const uint32_t d = 2;
            f.write(reinterpret_cast<const char *>(&d), 4);
            f.write(reinterpret_cast<const char *>(r), 8);
        }
        std::ofstream g(dir + "/b.fbin", std::ios::binary);
        const uint32_t hdr[2] = {3, 2};
        g.write(reinterpret_cast<const char *>(hdr), 8);
        g.write(reinterpret_cast<const char *>(rows), sizeof(rows));
        std::ofstream t(dir + "/trunc.fbin", std::ios::binary);
        t.write(reinterpret_cast<const char *>(hdr), 8);
        t.write(reinterpret_cast<const char *>(rows), 12);
    }
    for (const char *name : {"/b.fvecs", "/b.fbin"}) {
        auto m = load_vectors<float>(dir + name);
        CHECK(m.rows == 3 && m.cols == 2 && m(2, 1) == 3.f && m(1, 0) == 1.f);
        MappedVectors mv(dir + name);
        CHECK(mv.rows() == 3 && mv.dim() == 2 && mv.row(2)[1] == 3.f);
    }
    CHECK(throws([&] { load_vectors<float>(dir + "/trunc.fbin"); }));
    CHECK(throws([&] { MappedVectors m(dir + "/trunc.fbin"); }));
    CHECK(throws([&] { load_vectors<float>(dir + "/missing.fbin"); }));

    // recall: one query at the origin, GT top-2 = {0, 1}; id 2 is farther than rank 2
    const float q[2] = {0.f, 0.f};
    Matrix<uint32_t> gt;
    gt.rows = 1;
    gt.cols = 2;
    gt.data = {0, 1};
    RecallEvaluator ids_only(q, 1, 2, gt, 2, "");
    CHECK(ids_only.evaluate({1, 0}) == 1.0);
    CHECK(ids_only.evaluate({1, 1}) == 0.5);       // a repeated id counts once
    CHECK(ids_only.evaluate({2, UINT32_MAX}) == 0.0);
    // distance-aware: a row equal in distance to the GT radius counts as a hit
    {
        std::ofstream g(dir + "/d.fbin", std::ios::binary);
        const uint32_t hdr[2] = {4, 2};
        const float r4[4][2] = {{0.f, 0.f}, {1.f, 0.f}, {0.f, 3.f}, {0.f, -1.f}};
        g.write(reinterpret_cast<const char *>(hdr), 8);
        g.write(reinterpret_cast<const char *>(r4), sizeof(r4));
    }
    RecallEvaluator dist(q, 1, 2, gt, 2, dir + "/d.fbin");
    CHECK(dist.evaluate({0, 3}) == 1.0);   // id 3 is at distance 1 == radius
    CHECK(dist.evaluate({0, 2}) == 0.5);   // id 2 is at distance 9 > radius
    CHECK(dist.evaluate({0, 7}) == 0.5);   // out of range id is a miss
    // inner product: a row whose exact IP reaches the GT radius counts
    {
        const float qi[2] = {1.f, 0.f};
        Matrix<uint32_t> gti;
        gti.rows = 1;
        gti.cols = 1;
        gti.data = {1};  // id 1 = (1, 0): IP 1
        RecallEvaluator ip(qi, 1, 2, gti, 1, dir + "/d.fbin", 1);
        CHECK(ip.evaluate({1}) == 1.0);
        CHECK(ip.evaluate({3}) == 0.0);  // (0, -1): IP 0 < 1
        CHECK(throws([&] { RecallEvaluator bad(qi, 1, 2, gti, 1, "", 2); }));
    }
    Matrix<uint32_t> dup;
    dup.rows = 1;
    dup.cols = 2;
    dup.data = {1, 1};
    CHECK(throws([&] { RecallEvaluator e(q, 1, 2, dup, 2, ""); }));
    if (failures == 0) std::printf("bench headers: all checks passed\n");
    return failures == 0 ? 0 : 1;
}
