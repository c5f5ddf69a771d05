// mm.cu -- MatrixMarket coordinate reader (host code) behind cove_mm_read.
//
// Semantics of the reference loader (structural/include/structural/
// matrix_market.hpp:199-382): banner `%%MatrixMarket matrix coordinate
// <field> <symmetry>` (case-insensitive); lines that are empty or start
// with '%' are skipped; indices are 1-based; pattern entries are 1;
// symmetric / skew-symmetric files are expanded (skew negates the mirror);
// entries past the declared count are not read; each row is sorted by
// column, duplicates are summed and exact zeros dropped; values are parsed
// as double and cast to T.
//
// Layout: one pass over the file into COO arrays, a stable counting sort by
// row, then a stable sort of each row by column, so duplicates are summed in
// file order.
#include "cove_internal.cuh"

#include <algorithm>
#include <cctype>
#include <cerrno>
#include <climits>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <string>
#include <vector>

namespace cove {
namespace {

struct LineReader {
    FILE* f = nullptr;
    std::vector<char> buf;
    explicit LineReader(const char* path) : f(std::fopen(path, "rb")), buf(1 << 16) {}
    ~LineReader() {
        if (f) std::fclose(f);
    }
    // Next line without its newline; false at end of file.
    bool next(std::string& line) {
        line.clear();
        if (!f) return false;
        bool any = false;
        while (std::fgets(buf.data(), static_cast<int>(buf.size()), f)) {
            any = true;
            const size_t n = std::strlen(buf.data());
            if (n > 0 && buf[n - 1] == '\n') {
                line.append(buf.data(), n - 1);
                return true;
            }
            line.append(buf.data(), n);
        }
        return any;
    }
};

bool skip_line(const std::string& s) { return s.empty() || s[0] == '%'; }

int parse_field(const std::string& t) {
    if (t == "real") return COVE_MM_REAL;
    if (t == "integer") return COVE_MM_INTEGER;
    if (t == "complex") return COVE_MM_COMPLEX;
    if (t == "pattern") return COVE_MM_PATTERN;
    COVE_THROW(COVE_ERR_INVALID_INPUT, "unsupported MatrixMarket field: " + t);
}

int parse_symmetry(const std::string& t) {
    if (t == "general") return COVE_MM_GENERAL;
    if (t == "symmetric") return COVE_MM_SYMMETRIC;
    if (t == "skew-symmetric") return COVE_MM_SKEW_SYMMETRIC;
    if (t == "hermitian") return COVE_MM_HERMITIAN;
    COVE_THROW(COVE_ERR_INVALID_INPUT, "unsupported MatrixMarket symmetry: " + t);
}

int64_t parse_count(const char*& p, const char* what) {
    char* end = nullptr;
    errno = 0;
    const long long v = std::strtoll(p, &end, 10);
    if (end == p) COVE_THROW(COVE_ERR_INVALID_INPUT, std::string("invalid MatrixMarket ") + what);
    if (v < 0 || v > INT32_MAX || errno == ERANGE)
        COVE_THROW(COVE_ERR_INVALID_INPUT, std::string("MatrixMarket ") + what + " out of Index range");
    p = end;
    return v;
}

template <typename T>
void read_typed(const char* path, cove_mm_matrix* out) {
    LineReader in(path);
    if (!in.f) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, std::string("cannot open MatrixMarket file: ") + path);
    std::string line;
    if (!in.next(line)) COVE_THROW(COVE_ERR_INVALID_INPUT, std::string("empty MatrixMarket file: ") + path);
    std::string low(line);
    std::transform(low.begin(), low.end(), low.begin(),
                   [](unsigned char c) { return static_cast<char>(std::tolower(c)); });
    char b[64] = {}, o[64] = {}, fm[64] = {}, fl[64] = {}, sy[64] = {};
    if (std::sscanf(low.c_str(), "%63s %63s %63s %63s %63s", b, o, fm, fl, sy) != 5)
        COVE_THROW(COVE_ERR_INVALID_INPUT, std::string("invalid MatrixMarket header: ") + path);
    if (std::string(b) != "%%matrixmarket" || std::string(o) != "matrix" ||
        std::string(fm) != "coordinate")
        COVE_THROW(COVE_ERR_UNSUPPORTED, "only MatrixMarket coordinate matrices are supported");
    do {
        if (!in.next(line)) COVE_THROW(COVE_ERR_INVALID_INPUT, "missing MatrixMarket size line");
    } while (skip_line(line));
    const char* p = line.c_str();
    const int64_t rows = parse_count(p, "row count");
    const int64_t cols = parse_count(p, "column count");
    const int64_t declared = parse_count(p, "nnz count");
    const int field = parse_field(fl);
    const int sym = parse_symmetry(sy);
    if (field == COVE_MM_COMPLEX || sym == COVE_MM_HERMITIAN)
        COVE_THROW(COVE_ERR_UNSUPPORTED, "complex/hermitian MatrixMarket matrices need a complex loader");
    if (field == COVE_MM_PATTERN && sym == COVE_MM_SKEW_SYMMETRIC)
        COVE_THROW(COVE_ERR_INVALID_INPUT, "pattern skew-symmetric MatrixMarket matrices have no signed value");
    const bool mirror = sym != COVE_MM_GENERAL;

    std::vector<int32_t> er, ec;
    std::vector<T> ev;
    const size_t reserve = static_cast<size_t>(declared) * (mirror ? 2 : 1);
    er.reserve(reserve);
    ec.reserve(reserve);
    ev.reserve(reserve);
    int64_t read = 0;
    while (read < declared && in.next(line)) {
        if (skip_line(line)) continue;
        const char* q = line.c_str();
        char* end = nullptr;
        const long long r = std::strtoll(q, &end, 10);
        if (end == q) COVE_THROW(COVE_ERR_INVALID_INPUT, "invalid MatrixMarket row index");
        q = end;
        const long long c = std::strtoll(q, &end, 10);
        if (end == q) COVE_THROW(COVE_ERR_INVALID_INPUT, "invalid MatrixMarket column index");
        q = end;
        if (r <= 0 || r > INT32_MAX || c <= 0 || c > INT32_MAX)
            COVE_THROW(COVE_ERR_INVALID_INPUT, "MatrixMarket entry index out of Index range");
        T v = T(1);
        if (field != COVE_MM_PATTERN) {
            const double d = std::strtod(q, &end);
            if (end == q) COVE_THROW(COVE_ERR_INVALID_INPUT, "non-pattern MatrixMarket entry missing value");
            v = static_cast<T>(d);
        }
        if (r > rows || c > cols) COVE_THROW(COVE_ERR_INVALID_INPUT, "MatrixMarket entry index out of range");
        er.push_back(static_cast<int32_t>(r - 1));
        ec.push_back(static_cast<int32_t>(c - 1));
        ev.push_back(v);
        if (mirror && r != c) {
            er.push_back(static_cast<int32_t>(c - 1));
            ec.push_back(static_cast<int32_t>(r - 1));
            ev.push_back(sym == COVE_MM_SKEW_SYMMETRIC ? -v : v);
        }
        ++read;
    }
    if (read != declared) COVE_THROW(COVE_ERR_INVALID_INPUT, "MatrixMarket ended before all entries were read");

    // stable counting sort by row, then each row stably by column
    const size_t m = er.size();
    std::vector<int64_t> rp(static_cast<size_t>(rows) + 1, 0);
    for (size_t i = 0; i < m; ++i) ++rp[static_cast<size_t>(er[i]) + 1];
    std::partial_sum(rp.begin(), rp.end(), rp.begin());
    std::vector<int64_t> next(rp.begin(), rp.end() - 1);
    std::vector<int32_t> col(m);
    std::vector<T> val(m);
    for (size_t i = 0; i < m; ++i) {
        const int64_t d = next[static_cast<size_t>(er[i])]++;
        col[static_cast<size_t>(d)] = ec[i];
        val[static_cast<size_t>(d)] = ev[i];
    }
    std::vector<int64_t>().swap(next);
    std::vector<int32_t>().swap(er);
    std::vector<int32_t>().swap(ec);
    std::vector<T>().swap(ev);
    std::vector<int64_t> order;
    std::vector<int32_t> oc;
    std::vector<T> ov;
    int64_t w = 0;
    int64_t begin = 0;
    for (int64_t r = 0; r < rows; ++r) {
        const int64_t a = begin, e = rp[static_cast<size_t>(r) + 1];
        const int64_t n = e - a;
        order.resize(static_cast<size_t>(n));
        std::iota(order.begin(), order.end(), a);
        std::stable_sort(order.begin(), order.end(),
                         [&](int64_t i, int64_t j) { return col[static_cast<size_t>(i)] < col[static_cast<size_t>(j)]; });
        oc.resize(static_cast<size_t>(n));
        ov.resize(static_cast<size_t>(n));
        int64_t k = -1;  // coalesce duplicates (summed in file order)
        for (int64_t t = 0; t < n; ++t) {
            const int32_t c = col[static_cast<size_t>(order[static_cast<size_t>(t)])];
            const T v = val[static_cast<size_t>(order[static_cast<size_t>(t)])];
            if (k >= 0 && oc[static_cast<size_t>(k)] == c) {
                ov[static_cast<size_t>(k)] += v;
            } else {
                ++k;
                oc[static_cast<size_t>(k)] = c;
                ov[static_cast<size_t>(k)] = v;
            }
        }
        begin = e;
        rp[static_cast<size_t>(r)] = w;  // rows before r are final: reuse as output row_ptr
        for (int64_t t = 0; t <= k; ++t) {
            if (ov[static_cast<size_t>(t)] == T(0)) continue;  // exact zeros are dropped
            col[static_cast<size_t>(w)] = oc[static_cast<size_t>(t)];
            val[static_cast<size_t>(w)] = ov[static_cast<size_t>(t)];
            ++w;
        }
    }
    rp[static_cast<size_t>(rows)] = w;

    out->rows = static_cast<int32_t>(rows);
    out->cols = static_cast<int32_t>(cols);
    out->nnz = w;
    out->field = field;
    out->symmetry = sym;
    out->stored_entries = declared;
    out->expanded_entries = static_cast<int64_t>(m);
    out->coalesced_duplicates = static_cast<int64_t>(m) - w;
    out->row_ptr = static_cast<int64_t*>(std::malloc(sizeof(int64_t) * (static_cast<size_t>(rows) + 1)));
    out->col_idx = static_cast<int32_t*>(std::malloc(sizeof(int32_t) * std::max<int64_t>(w, 1)));
    out->values = std::malloc(sizeof(T) * std::max<int64_t>(w, 1));
    if (!out->row_ptr || !out->col_idx || !out->values) {
        cove_mm_free(out);
        COVE_THROW(COVE_ERR_OUT_OF_MEMORY, "host allocation for the MatrixMarket matrix failed");
    }
    std::memcpy(out->row_ptr, rp.data(), sizeof(int64_t) * (static_cast<size_t>(rows) + 1));
    std::memcpy(out->col_idx, col.data(), sizeof(int32_t) * static_cast<size_t>(w));
    std::memcpy(out->values, val.data(), sizeof(T) * static_cast<size_t>(w));
}

}  // namespace
}  // namespace cove

extern "C" {

cove_status cove_mm_read(const char* path, int32_t dtype, cove_mm_matrix* out) {
    return cove::guarded([&] {
        if (!path || !out) COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "null argument");
        *out = cove_mm_matrix{};
        out->dtype = dtype;
        if (dtype == COVE_F64) {
            cove::read_typed<double>(path, out);
        } else if (dtype == COVE_F32) {
            cove::read_typed<float>(path, out);
        } else {
            COVE_THROW(COVE_ERR_INVALID_ARGUMENT, "dtype must be COVE_F64 or COVE_F32");
        }
    });
}

void cove_mm_free(cove_mm_matrix* m) {
    if (!m) return;
    std::free(m->row_ptr);
    std::free(m->col_idx);
    std::free(m->values);
    m->row_ptr = nullptr;
    m->col_idx = nullptr;
    m->values = nullptr;
}

}  // extern "C"
