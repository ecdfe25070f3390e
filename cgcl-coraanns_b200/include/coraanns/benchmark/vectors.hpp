// Vector files used by the coraanns_search CLI and the recall evaluator.
//
// Formats (as the reference reads them, third_party/rabitq/.../utils/io.hpp:27-93 and
// include/coraanns/io/mapped_vectors.hpp): "*vecs" = per row a uint32 dimension followed by
// the row; anything else = uint32 rows, uint32 dim, then row-major data.
#pragma once

#include <sys/mman.h>
#include <sys/stat.h>
#include <fcntl.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace coraanns::bench {

template <typename T>
struct Matrix {
    std::vector<T> data;
    std::size_t rows = 0, cols = 0;
    T *row(std::size_t i) { return data.data() + i * cols; }
    const T *row(std::size_t i) const { return data.data() + i * cols; }
    T operator()(std::size_t i, std::size_t j) const { return data[i * cols + j]; }
};

inline bool ends_with_vecs(const std::string &path) {
    return path.size() > 4 && path.compare(path.size() - 4, 4, "vecs") == 0;
}

template <typename T>
Matrix<T> load_vectors(const std::string &path) {
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in) throw std::runtime_error("Cannot open vector file " + path);
    const std::size_t bytes = static_cast<std::size_t>(in.tellg());
    in.seekg(0);
    Matrix<T> m;
    if (ends_with_vecs(path)) {
        uint32_t dim = 0;
        in.read(reinterpret_cast<char *>(&dim), 4);
        if (!in || dim == 0) throw std::runtime_error("Invalid vecs header in " + path);
        const std::size_t rec = 4 + std::size_t{dim} * sizeof(T);
        if (bytes % rec) throw std::runtime_error("Truncated vecs file " + path);
        m.rows = bytes / rec;
        m.cols = dim;
        m.data.resize(m.rows * m.cols);
        in.seekg(0);
        for (std::size_t i = 0; i < m.rows; ++i) {
            uint32_t d = 0;
            in.read(reinterpret_cast<char *>(&d), 4);
            if (d != dim) throw std::runtime_error("Inconsistent vecs row length in " + path);
            in.read(reinterpret_cast<char *>(m.row(i)), dim * sizeof(T));
        }
    } else {
        uint32_t hdr[2] = {0, 0};
        in.read(reinterpret_cast<char *>(hdr), 8);
        if (!in || hdr[0] == 0 || hdr[1] == 0) throw std::runtime_error("Invalid bin header in " + path);
        m.rows = hdr[0];
        m.cols = hdr[1];
        if (bytes != 8 + m.rows * m.cols * sizeof(T))
            throw std::runtime_error("Size of " + path + " does not match its header");
        m.data.resize(m.rows * m.cols);
        in.read(reinterpret_cast<char *>(m.data.data()), m.data.size() * sizeof(T));
    }
    if (!in) throw std::runtime_error("Failed to read " + path);
    return m;
}

// Read-only, demand-paged view of a float vector file (either format), for exact distances
// of a few result rows without loading the base into RAM.
class MappedVectors {
  public:
    explicit MappedVectors(const std::string &path) {
        fd_ = ::open(path.c_str(), O_RDONLY);
        if (fd_ < 0) throw std::runtime_error("Cannot open " + path);
        struct stat st {};
        if (::fstat(fd_, &st) != 0 || st.st_size <= 8) {
            ::close(fd_);
            throw std::runtime_error("Empty or unreadable vector file " + path);
        }
        bytes_ = static_cast<std::size_t>(st.st_size);
        void *p = ::mmap(nullptr, bytes_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (p == MAP_FAILED) {
            ::close(fd_);
            throw std::runtime_error("Cannot mmap " + path);
        }
        base_ = static_cast<const uint8_t *>(p);
        if (ends_with_vecs(path)) {
            uint32_t d;
            std::memcpy(&d, base_, 4);
            dim_ = d;
            stride_ = 4 + dim_ * 4;
            offset_ = 4;
            if (dim_ == 0 || bytes_ % stride_) fail(path);
            rows_ = bytes_ / stride_;
        } else {
            uint32_t hdr[2];
            std::memcpy(hdr, base_, 8);
            rows_ = hdr[0];
            dim_ = hdr[1];
            stride_ = dim_ * 4;
            offset_ = 8;
            if (!rows_ || !dim_ || bytes_ != 8 + rows_ * stride_) fail(path);
        }
    }
    MappedVectors(const MappedVectors &) = delete;
    MappedVectors &operator=(const MappedVectors &) = delete;
    ~MappedVectors() {
        if (base_) ::munmap(const_cast<uint8_t *>(base_), bytes_);
        if (fd_ >= 0) ::close(fd_);
    }
    std::size_t rows() const { return rows_; }
    std::size_t dim() const { return dim_; }
    const uint8_t *mapping() const { return base_; }
    std::size_t row_stride_bytes() const { return stride_; }
    std::size_t data_offset_bytes() const { return offset_; }
    const float *row(std::size_t i) const {
        return reinterpret_cast<const float *>(base_ + offset_ + i * stride_);
    }

  private:
    [[noreturn]] void fail(const std::string &path) {
        ::munmap(const_cast<uint8_t *>(base_), bytes_);
        ::close(fd_);
        base_ = nullptr;
        fd_ = -1;
        throw std::runtime_error("Malformed vector file " + path);
    }
    int fd_ = -1;
    const uint8_t *base_ = nullptr;
    std::size_t bytes_ = 0, rows_ = 0, dim_ = 0, stride_ = 0, offset_ = 0;
};

}  // namespace coraanns::bench
