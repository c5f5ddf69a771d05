// convert.hpp -- host entry of the CSR -> BitBSR conversion
// (structural/include/structural/convert.hpp:13-165), same name and
// parameters.  The conversion runs on the GPU (the warp-direct 8x4
// converter of gpu_convert.cuh) and the result is copied back: block rows
// of 8 rows, distinct block columns ascending, bitmap bit = local_row * 4 +
// local_col, values in block then bit order, stored zeros dropped -- the
// reference's layout, bit for bit.  This build converts 8x4 blocks only;
// other positive block sizes raise an error.
#pragma once

#include "structural/gpu_convert.cuh"

#include <stdexcept>

namespace structural {

template <typename T>
BitBsrMatrix<T> convert_to_bitbsr(const CsrMatrix<T>& csr, Index block_rows, Index block_cols) {
    if (block_rows <= 0 || block_cols <= 0) throw std::runtime_error("BitBSR block sizes must be positive");
    if (block_rows != 8 || block_cols != 4) throw std::runtime_error("this build converts to 8x4 BitBSR blocks only");
    GpuBitBsrWorkspace<T> workspace;
    DeviceBitBsrMatrix<T> device;
    convert_to_bitbsr_gpu_warp_direct_8x4_device(csr, workspace, device);
    return device.to_host();
}

}  // namespace structural
