// Command-line options of the coraanns_search CLI.
//
// The options are declared once, as a table of specs (name, kind); one parser then turns
// argv into typed values in three passes: split the tokens into (key, value) pairs,
// reject keys the table does not name, and convert every value to its kind in table order.
// What users see is the reference's interface (include/coraanns/benchmark/options.hpp:11-169
// of the reference project), kept because scripts drive the CLI through it:
//   * `--key value` or `--key=value`; a bare word is "Unexpected positional argument: w";
//     a key followed by another option or by nothing is "Missing value for --key";
//   * a key given twice (or an empty key) is "Invalid or duplicate option --key";
//   * a key outside the table is "Unknown option --key";
//   * sizes are unsigned decimals without a sign ("Invalid integer for --key: text"); an
//     empty value (`--key=`) means "not given";
//   * booleans are true/false, 1/0, yes/no, on/off ("Invalid boolean for --key: text");
//   * --nprobes is a comma list of distinct values in [1, nlist], or the reference's default
//     grid clipped to nlist;
//   * --recall-base FILE may sit anywhere on the command line (recall.hpp:20-50) and is
//     taken out of argv before the positional arguments are read.
#pragma once

#include <cstddef>
#include <initializer_list>
#include <set>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace coraanns::bench {

enum class OptionKind { kSize, kBool, kText };

struct OptionSpec {
    const char *name;  // without the leading "--"
    OptionKind kind;
};

namespace detail {

inline bool looks_like_option(const char *word) {
    return word != nullptr && word[0] == '-' && word[1] == '-';
}

// Unsigned decimal covering the whole string; false on a sign, a stray character or overflow.
inline bool to_unsigned(const std::string &text, std::size_t &out) {
    if (text.empty()) return false;
    std::size_t v = 0;
    for (const char ch : text) {
        if (ch < '0' || ch > '9') return false;
        const std::size_t digit = static_cast<std::size_t>(ch - '0');
        if (v > (static_cast<std::size_t>(-1) - digit) / 10) return false;
        v = v * 10 + digit;
    }
    out = v;
    return true;
}

inline bool to_flag(const std::string &text, bool &out) {
    static const std::pair<const char *, bool> words[] = {
        {"true", true}, {"1", true}, {"yes", true}, {"on", true},
        {"false", false}, {"0", false}, {"no", false}, {"off", false}};
    for (const auto &w : words)
        if (text == w.first) {
            out = w.second;
            return true;
        }
    return false;
}

}  // namespace detail

class OptionTable {
  public:
    OptionTable(std::initializer_list<OptionSpec> specs) {
        for (const OptionSpec &s : specs) {
            Slot slot;
            slot.spec = s;
            slots_.push_back(slot);
        }
    }

    // argv[first, argc) must hold options only.
    void parse(int argc, char **argv, int first) {
        std::vector<std::pair<std::string, std::string>> pairs;
        std::set<std::string> seen;
        for (int i = first; i < argc; ++i) {  // pass 1: tokens -> (key, value)
            const std::string word(argv[i]);
            if (!detail::looks_like_option(argv[i]))
                throw std::invalid_argument("Unexpected positional argument: " + word);
            const std::string body = word.substr(2);
            const std::size_t eq = body.find('=');
            std::string key = body.substr(0, eq), value;
            if (eq != std::string::npos) {
                value = body.substr(eq + 1);
            } else if (i + 1 < argc && !detail::looks_like_option(argv[i + 1])) {
                value = argv[++i];
            } else {
                throw std::invalid_argument("Missing value for --" + key);
            }
            if (key.empty() || !seen.insert(key).second)
                throw std::invalid_argument("Invalid or duplicate option --" + key);
            pairs.emplace_back(std::move(key), std::move(value));
        }
        for (const auto &kv : pairs) {  // pass 2: every key must be in the table
            Slot *slot = find(kv.first);
            if (!slot) throw std::invalid_argument("Unknown option --" + kv.first);
            slot->given = true;
            slot->raw = kv.second;
        }
        for (Slot &slot : slots_) convert(slot);  // pass 3: typed values, table order
    }

    bool given(const std::string &name) const { return at(name).given; }

    std::size_t size(const std::string &name, std::size_t fallback) const {
        const Slot &s = at(name, OptionKind::kSize);
        return s.has_value ? s.number : fallback;
    }
    bool flag(const std::string &name, bool fallback) const {
        const Slot &s = at(name, OptionKind::kBool);
        return s.has_value ? s.truth : fallback;
    }
    std::string text(const std::string &name, const std::string &fallback) const {
        const Slot &s = at(name, OptionKind::kText);
        return s.given ? s.raw : fallback;
    }

  private:
    struct Slot {
        OptionSpec spec{"", OptionKind::kText};
        bool given = false, has_value = false, truth = false;
        std::size_t number = 0;
        std::string raw;
    };

    static void convert(Slot &s) {
        if (!s.given) return;
        const std::string key = s.spec.name;
        switch (s.spec.kind) {
            case OptionKind::kSize:
                if (s.raw.empty()) return;  // `--key=`: not given
                if (!detail::to_unsigned(s.raw, s.number))
                    throw std::invalid_argument("Invalid integer for --" + key + ": " + s.raw);
                break;
            case OptionKind::kBool:
                if (!detail::to_flag(s.raw, s.truth))
                    throw std::invalid_argument("Invalid boolean for --" + key + ": " + s.raw);
                break;
            case OptionKind::kText:
                break;
        }
        s.has_value = true;
    }

    Slot *find(const std::string &name) {
        for (Slot &s : slots_)
            if (name == s.spec.name) return &s;
        return nullptr;
    }
    const Slot &at(const std::string &name) const {
        for (const Slot &s : slots_)
            if (name == s.spec.name) return s;
        throw std::logic_error("option --" + name + " is not declared in the table");
    }
    const Slot &at(const std::string &name, OptionKind kind) const {
        const Slot &s = at(name);
        if (s.spec.kind != kind) throw std::logic_error("option --" + name + " read as another kind");
        return s;
    }

    std::vector<Slot> slots_;
};

// --nprobes: "a,b,c" with every value in [1, nlist] and no repeats; empty text gives the
// reference's default grid, clipped to nlist (nlist itself when nothing remains).
inline std::vector<std::size_t> parse_nprobes(const std::string &text, std::size_t nlist) {
    static const std::size_t kDefaultGrid[] = {40, 50, 60, 75, 95, 128, 180, 255, 400, 535, 775, 1400};
    std::vector<std::size_t> grid;
    if (text.empty()) {
        for (const std::size_t v : kDefaultGrid)
            if (v <= nlist) grid.push_back(v);
        if (grid.empty()) grid.push_back(nlist);
        return grid;
    }
    std::set<std::size_t> used;
    std::string item;
    for (std::size_t pos = 0; pos <= text.size(); ++pos) {
        if (pos < text.size() && text[pos] != ',') {
            item.push_back(text[pos]);
            continue;
        }
        const char lead = item.empty() ? '\0' : item.front();
        if (item.empty() || lead == '-' || lead == '+')
            throw std::invalid_argument("Invalid value in --nprobes: " + item);
        std::size_t v = 0;
        if (!detail::to_unsigned(item, v) || v == 0 || v > nlist)
            throw std::invalid_argument("Each nprobe must be in [1, nlist]; got: " + item);
        if (!used.insert(v).second) throw std::invalid_argument("Duplicate nprobe value: " + item);
        grid.push_back(v);
        item.clear();
    }
    return grid;
}

inline std::string join_values(const std::vector<std::size_t> &values) {
    std::string out;
    for (const std::size_t v : values) {
        if (!out.empty()) out += ',';
        out += std::to_string(v);
    }
    return out;
}

// Shapes of the query set, the ground truth and the index must agree before any search.
inline void validate_benchmark_shape(std::size_t query_rows, std::size_t query_dim,
                                     std::size_t gt_rows, std::size_t gt_dim,
                                     std::size_t index_dim, std::size_t topk, std::size_t rounds) {
    const auto n = [](std::size_t v) { return std::to_string(v); };
    const std::pair<bool, std::string> checks[] = {
        {topk == 0, "topk must be positive"},
        {rounds == 0, "rounds must be positive"},
        {query_rows == 0 || query_dim == 0, "The query set must not be empty"},
        {query_rows != gt_rows,
         "Query/ground-truth row mismatch: " + n(query_rows) + " vs " + n(gt_rows)},
        {query_dim != index_dim,
         "Query/index dimension mismatch: " + n(query_dim) + " vs " + n(index_dim)},
        {gt_dim < topk, "Ground truth has only " + n(gt_dim) +
                            " neighbors per query, fewer than topk=" + n(topk)},
    };
    for (const auto &c : checks)
        if (c.first) throw std::invalid_argument(c.second);
}

// Takes `--recall-base FILE` / `--recall-base=FILE` out of argv wherever it appears and
// returns FILE ("" when absent). The remaining words keep their order; argc shrinks.
inline std::string take_recall_base(int &argc, char **argv) {
    static const std::string kFlag = "--recall-base";
    std::string file;
    int hits = 0, kept = 1;
    for (int i = 1; i < argc; ++i) {
        const std::string word(argv[i]);
        const bool joined = word.compare(0, kFlag.size() + 1, kFlag + "=") == 0;
        if (word != kFlag && !joined) {
            argv[kept++] = argv[i];
            continue;
        }
        if (++hits > 1) throw std::invalid_argument("Duplicate --recall-base");
        if (joined) {
            file = word.substr(kFlag.size() + 1);
        } else {
            if (i + 1 >= argc || detail::looks_like_option(argv[i + 1]))
                throw std::invalid_argument("Missing file for --recall-base");
            file = argv[++i];
        }
        if (file.empty()) throw std::invalid_argument("Empty --recall-base");
    }
    argc = kept;
    argv[argc] = nullptr;
    if (hits && argc < 4)
        throw std::invalid_argument("--recall-base does not replace index/query/GT arguments");
    return file;
}

}  // namespace coraanns::bench
