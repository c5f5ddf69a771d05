// cove_codecs.cuh -- joint value-stream encoders.
#pragma once

#include "cove_convert.cuh"

namespace cove {

struct DictStreams {
    int64_t uniq = 0;  // distinct values, -1 if more than 65536
    int bits = 8;      // 8 or 16
    DevBuf codebook;   // T, first-occurrence order
    DevBuf kept_idx;   // uint8/uint16 per kept nnz
    DevBuf res_idx;    // uint8/uint16 per residual nnz
};

template <typename T>
void encode_bfp8(const SplitParts& sp, const uint8_t* is_out, DevBuf& q, DevBuf& scale,
                 cudaStream_t s);
template <typename T>
double select_abs_order_statistic(const T* vals, int64_t n, int64_t idx, cudaStream_t s);
template <typename T>
void encode_bfp8_outlier(const SplitParts& sp, int32_t nbr, double fraction, DevBuf& q,
                         DevBuf& scale, DevBuf& orow, DevBuf& ocol, DevBuf& oval,
                         int64_t* num_out, double* threshold, cudaStream_t s);
template <typename T>
void encode_res_bf16(const SplitParts& sp, DevBuf& out, cudaStream_t s);
// Returns the distinct-value count (-1 if above 65536); fills codes when
// build_codes and the count fits.
template <typename T>
int64_t encode_dict(const SplitParts& sp, bool build_codes, DictStreams& out, cudaStream_t s);

}  // namespace cove
