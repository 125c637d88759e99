// Matrix Market coordinate reader into canonical CSR, behaviour-compatible with the
// reference's loadMatrixMarket (src/format/matrix_market.cpp:30-103): the same accepted
// headers (coordinate real/integer/pattern, general/symmetric), 1-based indices, pattern
// entries of weight 1, symmetric off-diagonals mirrored, every row's entries kept in file
// order before makeCanonicalCsr sums duplicates, and the same error messages.
// Implementation: one pass over the file into (row, col, value) triplets parsed with
// strtoull/strtof, then a stable counting sort by row.
#include "common.hpp"
#include "format/csr.h"

#include <cctype>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <string>

namespace tcc {
CsrMatrix canonicalCsr(std::uint32_t rows, std::uint32_t cols, std::uint32_t nnz, const std::uint32_t* offsets,
                       const std::uint32_t* sources, const float* values, unsigned threads);
namespace {

class LineReader {
  public:
    explicit LineReader(const std::string& path) : file_(std::fopen(path.c_str(), "rb")) {}
    ~LineReader() {
        if (file_)
            std::fclose(file_);
    }
    bool ok() const { return file_ != nullptr; }
    // Next line without the trailing newline; false at end of file.
    bool next(std::string& line) {
        line.clear();
        int ch;
        bool any = false;
        while ((ch = std::fgetc(file_)) != EOF) {
            any = true;
            if (ch == '\n')
                return true;
            line.push_back(static_cast<char>(ch));
        }
        return any;
    }
    // Next line that is neither blank nor a comment.
    bool nextData(std::string& line) {
        while (next(line)) {
            const auto first = line.find_first_not_of(" \t\r");
            if (first != std::string::npos && line[first] != '%')
                return true;
        }
        return false;
    }

  private:
    std::FILE* file_;
};

std::string lower(std::string s) {
    for (auto& c : s)
        c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
    return s;
}

// Parse an unsigned integer token; returns false if none is present.
bool parseU64(const char*& p, std::uint64_t& out) {
    while (*p == ' ' || *p == '\t' || *p == '\r')
        ++p;
    if (*p == '\0')
        return false;
    char* end = nullptr;
    errno = 0;
    out = std::strtoull(p, &end, 10);
    if (end == p)
        return false;
    p = end;
    return true;
}

bool parseFloat(const char*& p, float& out) {
    while (*p == ' ' || *p == '\t' || *p == '\r')
        ++p;
    if (*p == '\0')
        return false;
    char* end = nullptr;
    out = std::strtof(p, &end);
    if (end == p)
        return false;
    p = end;
    return true;
}

} // namespace

MtxMatrix loadMatrixMarketFile(const std::string& path) {
    LineReader in(path);
    if (!in.ok())
        throw std::runtime_error("cannot open Matrix Market file: " + path);
    std::string line;
    in.next(line);
    char tok[5][64] = {};
    std::sscanf(line.c_str(), "%63s %63s %63s %63s %63s", tok[0], tok[1], tok[2], tok[3], tok[4]);
    const std::string banner = lower(tok[0]), object = lower(tok[1]), storage = lower(tok[2]),
                      field = lower(tok[3]), symmetry = lower(tok[4]);
    if (banner != "%%matrixmarket" || object != "matrix" || storage != "coordinate" ||
        (field != "real" && field != "integer" && field != "pattern") ||
        (symmetry != "general" && symmetry != "symmetric"))
        throw std::runtime_error("expected a coordinate real/integer/pattern general/symmetric Matrix Market file");
    const bool pattern = field == "pattern", symmetric = symmetry == "symmetric";
    if (!in.nextData(line))
        throw std::runtime_error("missing Matrix Market dimensions");
    constexpr std::uint64_t max = std::numeric_limits<std::uint32_t>::max();
    std::uint64_t rows64 = 0, cols64 = 0, entries64 = 0;
    {
        const char* p = line.c_str();
        if (!parseU64(p, rows64) || !parseU64(p, cols64) || !parseU64(p, entries64) || !rows64 || !cols64 ||
            rows64 > max || cols64 > max || entries64 > max || (symmetric && rows64 != cols64))
            throw std::runtime_error("invalid or unsupported Matrix Market dimensions");
    }
    const auto rows = static_cast<std::uint32_t>(rows64);
    const auto cols = static_cast<std::uint32_t>(cols64);
    std::vector<std::uint32_t> tr, tc;
    std::vector<float> tv;
    tr.reserve(entries64);
    tc.reserve(entries64);
    tv.reserve(entries64);
    std::uint64_t expanded = 0;
    auto push = [&](std::uint32_t r, std::uint32_t c, float v) {
        if (++expanded > max)
            throw std::overflow_error("Matrix Market matrix exceeds uint32 CSR offsets");
        tr.push_back(r);
        tc.push_back(c);
        tv.push_back(v);
    };
    for (std::uint64_t i = 0; i < entries64; ++i) {
        if (!in.nextData(line))
            throw std::runtime_error("truncated Matrix Market file");
        const char* p = line.c_str();
        std::uint64_t row = 0, col = 0;
        float value = 1.0f;
        if (!parseU64(p, row) || !parseU64(p, col) || !row || row > rows || !col || col > cols ||
            (!pattern && !parseFloat(p, value)) || !std::isfinite(value))
            throw std::runtime_error("invalid Matrix Market entry");
        push(static_cast<std::uint32_t>(row - 1), static_cast<std::uint32_t>(col - 1), value);
        if (symmetric && row != col)
            push(static_cast<std::uint32_t>(col - 1), static_cast<std::uint32_t>(row - 1), value);
    }
    // Stable counting sort by row keeps every row's entries in file order.
    std::vector<std::uint32_t> offsets(std::size_t(rows) + 1, 0);
    for (std::uint32_t r : tr)
        ++offsets[std::size_t(r) + 1];
    for (std::size_t r = 1; r < offsets.size(); ++r)
        offsets[r] += offsets[r - 1];
    std::vector<std::uint32_t> columns(expanded), cursor(offsets.begin(), offsets.end() - 1);
    std::vector<float> values(expanded);
    for (std::size_t e = 0; e < tr.size(); ++e) {
        const auto at = cursor[tr[e]]++;
        columns[at] = tc[e];
        values[at] = tv[e];
    }
    MtxMatrix out{rows, cols, {}};
    out.csr = canonicalCsr(rows, cols, static_cast<std::uint32_t>(expanded), offsets.data(), columns.data(),
                           values.data(), 0);
    return out;
}

} // namespace tcc

MtxMatrix loadMatrixMarket(const std::string& path) { return tcc::loadMatrixMarketFile(path); }
