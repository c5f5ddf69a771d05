// csr.hpp -- host CSR container of the structural:: API
// (structural/include/structural/csr.hpp:11-50): same members and checks.
#pragma once

#include "structural/types.hpp"

#include <stdexcept>
#include <vector>

namespace structural {

template <typename T>
struct CsrMatrix {
    Index rows = 0;
    Index cols = 0;
    std::vector<Offset> row_ptr;
    std::vector<Index> col_idx;
    std::vector<T> values;

    Offset nnz() const { return static_cast<Offset>(values.size()); }

    void validate() const {
        if (rows < 0 || cols < 0) throw std::runtime_error("CSR dimensions must be non-negative");
        if (static_cast<Index>(row_ptr.size()) != rows + 1) {
            throw std::runtime_error("CSR row_ptr size must be rows + 1");
        }
        if (col_idx.size() != values.size()) throw std::runtime_error("CSR col_idx and values sizes differ");
        if (!row_ptr.empty() && row_ptr.front() != 0) throw std::runtime_error("CSR row_ptr must start at zero");
        for (Index r = 0; r < rows; ++r) {
            if (row_ptr[r] > row_ptr[r + 1]) throw std::runtime_error("CSR row_ptr must be monotonic");
        }
        if (!row_ptr.empty() && row_ptr.back() != nnz()) {
            throw std::runtime_error("CSR row_ptr.back must equal nnz");
        }
        for (const Index c : col_idx) {
            if (c < 0 || c >= cols) throw std::runtime_error("CSR column index out of range");
        }
    }
};

}  // namespace structural
