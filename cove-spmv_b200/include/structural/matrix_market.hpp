// matrix_market.hpp -- MatrixMarket loading of the structural:: API
// (structural/include/structural/matrix_market.hpp:18-92, 327-389): the same
// enums, info/result types and entry points, read by cove_mm_read.
// Host-only: include it from plain C++ and link libcove_b200.
#pragma once

#include "cove_b200.h"
#include "structural/csr.hpp"

#include <climits>
#include <cstring>
#include <stdexcept>
#include <string>
#include <type_traits>

namespace structural {

enum class MatrixMarketField { Real, Integer, Complex, Pattern };
enum class MatrixMarketSymmetry { General, Symmetric, SkewSymmetric, Hermitian };

inline const char* to_string(MatrixMarketField field) {
    switch (field) {
        case MatrixMarketField::Real: return "real";
        case MatrixMarketField::Integer: return "integer";
        case MatrixMarketField::Complex: return "complex";
        case MatrixMarketField::Pattern: return "pattern";
    }
    return "unknown";
}

inline const char* to_string(MatrixMarketSymmetry symmetry) {
    switch (symmetry) {
        case MatrixMarketSymmetry::General: return "general";
        case MatrixMarketSymmetry::Symmetric: return "symmetric";
        case MatrixMarketSymmetry::SkewSymmetric: return "skew-symmetric";
        case MatrixMarketSymmetry::Hermitian: return "hermitian";
    }
    return "unknown";
}

struct MatrixMarketInfo {
    Index rows = 0;
    Index cols = 0;
    Offset nnz_file = 0;
    MatrixMarketField field = MatrixMarketField::Real;
    MatrixMarketSymmetry symmetry = MatrixMarketSymmetry::General;

    bool is_pattern() const { return field == MatrixMarketField::Pattern; }
    bool requires_mirror_expansion() const { return symmetry != MatrixMarketSymmetry::General; }
    bool mirrors_with_negation() const { return symmetry == MatrixMarketSymmetry::SkewSymmetric; }
};

template <typename T>
struct MatrixMarketLoadResult {
    MatrixMarketInfo info;
    CsrMatrix<T> matrix;
    Offset stored_entries = 0;
    Offset expanded_entries = 0;
    Offset coalesced_duplicates = 0;
};

template <typename T>
MatrixMarketLoadResult<T> read_matrix_market_with_info(const std::string& path) {
    static_assert(std::is_same_v<T, double> || std::is_same_v<T, float>,
                  "the MatrixMarket loader reads float and double");
    cove_mm_matrix m{};
    if (cove_mm_read(path.c_str(), std::is_same_v<T, double> ? COVE_F64 : COVE_F32, &m) != COVE_OK) {
        throw std::runtime_error(cove_last_error());
    }
    struct Release {
        cove_mm_matrix* m;
        ~Release() { cove_mm_free(m); }
    } release{&m};
    if (m.expanded_entries > INT_MAX) {
        throw std::runtime_error("MatrixMarket matrix exceeds the int32 offsets of CsrMatrix");
    }
    MatrixMarketLoadResult<T> r;
    r.info.rows = m.rows;
    r.info.cols = m.cols;
    r.info.nnz_file = static_cast<Offset>(m.stored_entries);
    r.info.field = static_cast<MatrixMarketField>(m.field);
    r.info.symmetry = static_cast<MatrixMarketSymmetry>(m.symmetry);
    r.matrix.rows = m.rows;
    r.matrix.cols = m.cols;
    r.matrix.row_ptr.assign(m.row_ptr, m.row_ptr + m.rows + 1);
    r.matrix.col_idx.assign(m.col_idx, m.col_idx + m.nnz);
    r.matrix.values.resize(static_cast<size_t>(m.nnz));
    if (m.nnz > 0) std::memcpy(r.matrix.values.data(), m.values, sizeof(T) * static_cast<size_t>(m.nnz));
    r.stored_entries = static_cast<Offset>(m.stored_entries);
    r.expanded_entries = static_cast<Offset>(m.expanded_entries);
    r.coalesced_duplicates = static_cast<Offset>(m.coalesced_duplicates);
    return r;
}

template <typename T>
CsrMatrix<T> read_matrix_market(const std::string& path) {
    return read_matrix_market_with_info<T>(path).matrix;
}

}  // namespace structural
