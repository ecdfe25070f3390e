// Command-line options of the coraanns_search CLI, with the reference's rules
// (include/coraanns/benchmark/options.hpp:11-169): `--key value` or `--key=value`, strict
// known-key check, duplicates rejected, unsigned integers without sign, booleans
// true/false/1/0/yes/no/on/off, nprobe lists of distinct values in [1, nlist].
#pragma once

#include <algorithm>
#include <cstddef>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace coraanns::bench {

inline bool is_option(const char *text) { return text && text[0] == '-' && text[1] == '-'; }

class CliOptions {
  public:
    CliOptions(int argc, char **argv, int begin) {
        for (int i = begin; i < argc; ++i) {
            std::string arg(argv[i]);
            if (arg.rfind("--", 0) != 0)
                throw std::invalid_argument("Unexpected positional argument: " + arg);
            arg.erase(0, 2);
            std::string key, value;
            const auto eq = arg.find('=');
            if (eq != std::string::npos) {
                key = arg.substr(0, eq);
                value = arg.substr(eq + 1);
            } else {
                key = arg;
                if (i + 1 >= argc || is_option(argv[i + 1]))
                    throw std::invalid_argument("Missing value for --" + key);
                value = argv[++i];
            }
            if (key.empty() || values_.count(key))
                throw std::invalid_argument("Invalid or duplicate option --" + key);
            values_[key] = value;
        }
    }
    void require_known(const std::vector<std::string> &known) const {
        for (const auto &kv : values_)
            if (std::find(known.begin(), known.end(), kv.first) == known.end())
                throw std::invalid_argument("Unknown option --" + kv.first);
    }
    bool contains(const std::string &key) const { return values_.count(key) != 0; }
    std::string get(const std::string &key, const std::string &fallback) const {
        const auto it = values_.find(key);
        return it == values_.end() ? fallback : it->second;
    }
    std::size_t get_size(const std::string &key, std::size_t fallback) const {
        const std::string text = get(key, "");
        if (text.empty()) return fallback;
        if (text.front() == '-' || text.front() == '+')
            throw std::invalid_argument("Invalid integer for --" + key + ": " + text);
        std::size_t used = 0;
        unsigned long long v = 0;
        try {
            v = std::stoull(text, &used);
        } catch (const std::exception &) {
            throw std::invalid_argument("Invalid integer for --" + key + ": " + text);
        }
        if (used != text.size()) throw std::invalid_argument("Invalid integer for --" + key + ": " + text);
        return static_cast<std::size_t>(v);
    }
    bool get_bool(const std::string &key, bool fallback) const {
        const std::string t = get(key, fallback ? "true" : "false");
        if (t == "true" || t == "1" || t == "yes" || t == "on") return true;
        if (t == "false" || t == "0" || t == "no" || t == "off") return false;
        throw std::invalid_argument("Invalid boolean for --" + key + ": " + t);
    }

  private:
    std::map<std::string, std::string> values_;
};

inline std::vector<std::size_t> parse_nprobes(const std::string &text, std::size_t nlist) {
    std::vector<std::size_t> out;
    if (text.empty()) {
        for (std::size_t v : {40, 50, 60, 75, 95, 128, 180, 255, 400, 535, 775, 1400})
            if (v <= nlist) out.push_back(v);
        if (out.empty()) out.push_back(nlist);
        return out;
    }
    std::size_t begin = 0;
    while (true) {
        const auto comma = text.find(',', begin);
        const std::string tok = text.substr(begin, comma == std::string::npos ? std::string::npos : comma - begin);
        if (tok.empty() || tok.front() == '-' || tok.front() == '+')
            throw std::invalid_argument("Invalid value in --nprobes: " + tok);
        std::size_t used = 0;
        unsigned long long v = 0;
        try {
            v = std::stoull(tok, &used);
        } catch (const std::exception &) {
            throw std::invalid_argument("Invalid value in --nprobes: " + tok);
        }
        if (used != tok.size() || v == 0 || v > nlist)
            throw std::invalid_argument("Each nprobe must be in [1, nlist]; got: " + tok);
        if (std::find(out.begin(), out.end(), v) != out.end())
            throw std::invalid_argument("Duplicate nprobe value: " + tok);
        out.push_back(static_cast<std::size_t>(v));
        if (comma == std::string::npos) break;
        begin = comma + 1;
    }
    return out;
}

inline std::string join_values(const std::vector<std::size_t> &v) {
    std::string s;
    for (std::size_t i = 0; i < v.size(); ++i) s += (i ? "," : "") + std::to_string(v[i]);
    return s;
}

inline void validate_benchmark_shape(std::size_t query_rows, std::size_t query_dim,
                                     std::size_t gt_rows, std::size_t gt_dim,
                                     std::size_t index_dim, std::size_t topk, std::size_t rounds) {
    if (topk == 0) throw std::invalid_argument("topk must be positive");
    if (rounds == 0) throw std::invalid_argument("rounds must be positive");
    if (query_rows == 0 || query_dim == 0) throw std::invalid_argument("The query set must not be empty");
    if (query_rows != gt_rows)
        throw std::invalid_argument("Query/ground-truth row mismatch: " + std::to_string(query_rows) +
                                    " vs " + std::to_string(gt_rows));
    if (query_dim != index_dim)
        throw std::invalid_argument("Query/index dimension mismatch: " + std::to_string(query_dim) +
                                    " vs " + std::to_string(index_dim));
    if (gt_dim < topk)
        throw std::invalid_argument("Ground truth has only " + std::to_string(gt_dim) +
                                    " neighbors per query, fewer than topk=" + std::to_string(topk));
}

// Removes `--recall-base FILE` / `--recall-base=FILE` from argv (recall.hpp:20-50).
inline std::string take_recall_base(int &argc, char **argv) {
    std::string base;
    bool found = false;
    int out = 1;
    for (int i = 1; i < argc; ++i) {
        const std::string a(argv[i]);
        if (a == "--recall-base" || a.rfind("--recall-base=", 0) == 0) {
            if (found) throw std::invalid_argument("Duplicate --recall-base");
            found = true;
            if (a == "--recall-base") {
                if (i + 1 == argc || std::string(argv[i + 1]).rfind("--", 0) == 0)
                    throw std::invalid_argument("Missing file for --recall-base");
                base = argv[++i];
            } else {
                base = a.substr(14);
            }
            if (base.empty()) throw std::invalid_argument("Empty --recall-base");
        } else {
            argv[out++] = argv[i];
        }
    }
    argc = out;
    argv[argc] = nullptr;
    if (found && argc < 4)
        throw std::invalid_argument("--recall-base does not replace index/query/GT arguments");
    return base;
}

}  // namespace coraanns::bench
