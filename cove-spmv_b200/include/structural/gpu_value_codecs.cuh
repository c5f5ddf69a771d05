// gpu_value_codecs.cuh -- payload builders of the BitBSR-only value codecs
// and the exact-value histogram behind the auto_lossless choice, with the
// reference's names (structural/include/structural/gpu_value_codecs.cuh:
// 20-700, value_compression.hpp:105-198, selector main_gpu_spmv.cu:127-174).
// The payloads are the plan fields run_bitbsr_spmv_once decodes; the
// encodings (cell bit order, tile packing, bf16/fp16 rounding, BFP scales)
// are the reference's formats, bit for bit (BFP8 with global outliers
// included), and so are the k-means
// codebooks of k256 and global log-k-means (value_compression.hpp:265-341,
// 343-422, 452-497; gpu_value_codecs.cuh:693-744), whose steps are kept
// in the same order so the same libm gives the same doubles.
#pragma once

#include "structural/bitbsr.hpp"
#include "structural/gpu_convert.cuh"
#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"
#include "structural/value_compression.hpp"

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace structural {

struct DeviceExactValueHistogram {
    Offset nnz = 0;
    Offset num_blocks = 0;
    std::size_t raw_payload_bytes = 0;
    int unique_count = 0;
    bool unique_overflow = false;
    bool all_one = false;
    bool const_c = false;
    bool sign2 = false;
    bool sign2_scale = false;
    std::size_t const_c_payload_bytes = 0;
    std::size_t sign2_payload_bytes = 0;
    std::size_t sign2_scale_payload_bytes = 0;
    std::size_t dict2_payload_bytes = 0;
    std::size_t dict4_payload_bytes = 0;
    std::size_t dict16_payload_bytes = 0;
    std::size_t dict256_u8_payload_bytes = 0;
    std::size_t dict65536_u16_payload_bytes = 0;
};

// Distinct-value statistics of a device BitBSR matrix and each lossless
// codec's payload size.  unique_count counts up to 65537 (then
// unique_overflow is set).
template <typename T>
DeviceExactValueHistogram build_device_exact_value_histogram(const DeviceBitBsrMatrix<T>& bitbsr,
                                                             float* device_ms = nullptr) {
    gpu_detail::CudaEventTimer timer(device_ms);
    DeviceExactValueHistogram h;
    h.nnz = bitbsr.nnz;
    h.num_blocks = bitbsr.num_blocks;
    h.raw_payload_bytes = static_cast<std::size_t>(bitbsr.nnz) * sizeof(T);
    h.sign2_payload_bytes = static_cast<std::size_t>(bitbsr.num_blocks) * 4;
    h.const_c_payload_bytes = bitbsr.nnz > 0 ? sizeof(T) : 0;
    h.sign2_scale_payload_bytes = bitbsr.nnz > 0 ? h.sign2_payload_bytes + sizeof(T) : 0;
    if (bitbsr.nnz > 0) {
        std::vector<T> values(static_cast<size_t>(bitbsr.nnz));
        thrust::copy(bitbsr.values.begin(), bitbsr.values.end(), values.begin());
        const auto u = sorted_unique_values(values, 65536);
        h.unique_count = static_cast<int>(u.size());
        h.unique_overflow = u.size() > 65536;
        if (u.size() == 1) {
            h.const_c = true;
            h.all_one = u[0] == T(1);
        } else if (u.size() == 2) {
            h.sign2 = u[0] == T(-1) && u[1] == T(1);
            h.sign2_scale = u[0] != T(0) && u[0] == -u[1];
        }
    }
    auto dict_bytes = [&](int words) {
        return static_cast<std::size_t>(bitbsr.num_blocks) * words * 4 +
               static_cast<std::size_t>(h.unique_count) * sizeof(T);
    };
    h.dict2_payload_bytes = dict_bytes(1);
    h.dict4_payload_bytes = dict_bytes(2);
    h.dict16_payload_bytes = dict_bytes(4);
    h.dict256_u8_payload_bytes = dict_bytes(8);
    h.dict65536_u16_payload_bytes = dict_bytes(16);
    gpu_detail::finish(timer, device_ms);
    return h;
}

namespace cove {

// The smallest exact codec whose payload beats the raw values, as the
// operator's codec kind.  The reference keeps this choice inside its CLI
// (select_auto_lossless_value_codec, main_gpu_spmv.cu:127-174, file-local),
// so it lives in this shim's own namespace: reference sources that define
// theirs still compile against the shim.
inline BitBsrValueCodecKind8x4 select_auto_lossless_value_codec(const DeviceExactValueHistogram& h) {
    using K = BitBsrValueCodecKind8x4;
    if (h.nnz == 0) return K::Raw;
    auto saves = [&](std::size_t bytes) { return bytes < h.raw_payload_bytes; };
    if (h.all_one && saves(0)) return K::ImplicitOne;
    if (h.const_c && saves(h.const_c_payload_bytes)) return K::ConstC;
    if (h.sign2 && saves(h.sign2_payload_bytes)) return K::Sign2;
    if (h.sign2_scale && saves(h.sign2_scale_payload_bytes)) return K::Sign2Scale;
    if (h.unique_count <= 2 && saves(h.dict2_payload_bytes)) return K::Dict2;
    if (h.unique_count <= 4 && saves(h.dict4_payload_bytes)) return K::Unique4;
    if (h.unique_count <= 16 && saves(h.dict16_payload_bytes)) return K::Unique16;
    if (h.unique_count <= 256 && saves(h.dict256_u8_payload_bytes)) return K::Dict256U8;
    if (!h.unique_overflow && h.unique_count <= 65536 && saves(h.dict65536_u16_payload_bytes))
        return K::Dict65536U16;
    return K::Raw;
}

}  // namespace cove

// ---- per-cell walk ---------------------------------------------------------------

namespace codec_detail {
// f(block, bit, value_index) for every stored cell, blocks in order, bits ascending
template <typename T, typename F>
void for_each_cell(const BitBsrMatrix<T>& m, F&& f) {
    for (Offset b = 0; b < m.num_blocks(); ++b) {
        const std::uint32_t bm = m.bitmap_words[b];
        Offset k = m.block_val_ptr[b];
        for (int bit = 0; bit < 32; ++bit)
            if (bm & (1u << bit)) f(b, bit, k++);
    }
}
}  // namespace codec_detail

// ---- constant and sign codecs --------------------------------------------------

template <typename T>
T build_const_c_value(const BitBsrMatrix<T>& bitbsr) {
    bitbsr.validate();
    if (bitbsr.values.empty()) throw std::runtime_error("const_c value codec requires at least one value");
    for (const T v : bitbsr.values)
        if (v != bitbsr.values.front())
            throw std::runtime_error("const_c value codec requires every stored value to equal C");
    return bitbsr.values.front();
}

template <typename T>
void validate_implicit_one_values(const std::vector<T>& values) {
    for (const T v : values)
        if (v != T(1)) throw std::runtime_error("all_one value codec requires every stored value to be 1");
}

template <typename T>
struct Sign2ScaleTile32ValueCodec {
    T scale = T{1};
    std::vector<std::uint32_t> sign_masks;
    std::size_t payload_bytes() const { return sign_masks.size() * 4 + sizeof(T); }
};

// One word per block: cell bit set where the value is +1 (else it must be -1).
template <typename T>
std::vector<std::uint32_t> build_sign2_tile32_masks(const BitBsrMatrix<T>& bitbsr) {
    bitbsr.validate();
    std::vector<std::uint32_t> masks(static_cast<size_t>(bitbsr.num_blocks()), 0);
    codec_detail::for_each_cell(bitbsr, [&](Offset b, int bit, Offset k) {
        const T v = bitbsr.values[k];
        if (v == T(1)) masks[b] |= 1u << bit;
        else if (v != T(-1)) throw std::runtime_error("sign2 value codec requires values in {-1, +1}");
    });
    return masks;
}

template <typename T>
Sign2ScaleTile32ValueCodec<T> build_sign2_scale_tile32_value_codec(const BitBsrMatrix<T>& bitbsr) {
    bitbsr.validate();
    const auto u = sorted_unique_values(bitbsr.values, 2);
    if (u.size() != 2) throw std::runtime_error("sign2_scale value codec requires exactly two values");
    if (u[0] == T(0) || u[0] != -u[1]) throw std::runtime_error("sign2_scale value codec requires values in {-C, +C}");
    Sign2ScaleTile32ValueCodec<T> c;
    c.scale = u[1];
    c.sign_masks.assign(static_cast<size_t>(bitbsr.num_blocks()), 0);
    codec_detail::for_each_cell(bitbsr, [&](Offset b, int bit, Offset k) {
        if (bitbsr.values[k] == u[1]) c.sign_masks[b] |= 1u << bit;
    });
    return c;
}

// ---- tile codes ------------------------------------------------------------------

template <int BitsPerCode, typename T>
std::vector<std::uint32_t> build_tile_code_words_from_value_ids(const BitBsrMatrix<T>& bitbsr,
                                                                const std::vector<std::uint32_t>& value_ids) {
    static_assert(BitsPerCode == 1 || BitsPerCode == 2 || BitsPerCode == 4 || BitsPerCode == 8 ||
                      BitsPerCode == 16,
                  "tile codec supports 1, 2, 4, 8, or 16 bits per 8x4 cell");
    bitbsr.validate();
    if (value_ids.size() != bitbsr.values.size()) throw std::runtime_error("tile value codec id count mismatch");
    constexpr int kWords = BitsPerCode;  // 32 cells x BitsPerCode bits = BitsPerCode words
    constexpr int kPerWord = 32 / BitsPerCode;
    std::vector<std::uint32_t> words(static_cast<size_t>(bitbsr.num_blocks()) * kWords, 0);
    codec_detail::for_each_cell(bitbsr, [&](Offset b, int bit, Offset k) {
        const std::uint32_t id = value_ids[static_cast<size_t>(k)];
        if (BitsPerCode < 32 && id >= (1u << BitsPerCode))
            throw std::runtime_error("tile value codec id does not fit in tile field");
        words[static_cast<size_t>(b) * kWords + bit / kPerWord] |= id << ((bit % kPerWord) * BitsPerCode);
    });
    return words;
}

template <int BitsPerCode, typename T>
struct TileCodeValueCodec {
    std::vector<T> codebook;
    std::vector<std::uint32_t> value_ids;
    std::vector<std::uint32_t> tile_code_words;
    bool exact = true;
    std::size_t payload_bytes() const { return tile_code_words.size() * 4 + codebook.size() * sizeof(T); }
};

// Exact dictionary: codebook = ascending distinct values, id = rank.
template <int BitsPerCode, typename T>
TileCodeValueCodec<BitsPerCode, T> build_exact_tile_code_value_codec(const BitBsrMatrix<T>& bitbsr,
                                                                     int max_codebook_size, const char* name) {
    TileCodeValueCodec<BitsPerCode, T> c;
    c.codebook = sorted_unique_values(bitbsr.values, max_codebook_size);
    if (static_cast<int>(c.codebook.size()) > max_codebook_size)
        throw std::runtime_error(std::string(name) + " value codec requires fewer distinct values");
    std::unordered_map<T, std::uint32_t> rank;
    for (size_t i = 0; i < c.codebook.size(); ++i) rank.emplace(c.codebook[i], static_cast<std::uint32_t>(i));
    c.value_ids.resize(bitbsr.values.size());
    for (size_t i = 0; i < bitbsr.values.size(); ++i) {
        const auto it = rank.find(bitbsr.values[i]);
        if (it == rank.end()) throw std::runtime_error(std::string(name) + " exact value was not found in codebook");
        c.value_ids[i] = it->second;
    }
    c.tile_code_words = build_tile_code_words_from_value_ids<BitsPerCode>(bitbsr, c.value_ids);
    return c;
}

template <typename T> struct Dict2Tile32ValueCodec : TileCodeValueCodec<1, T> {};
template <typename T> struct Unique4Tile64ValueCodec : TileCodeValueCodec<2, T> {};
template <typename T> struct Unique16Tile128ValueCodec : TileCodeValueCodec<4, T> {};
template <typename T> struct Dict256Tile256ValueCodec : TileCodeValueCodec<8, T> {};
template <typename T> struct Dict65536Tile512ValueCodec : TileCodeValueCodec<16, T> {};

namespace codec_detail {
template <typename Out, int Bits, typename T>
Out named_tile_codec(const BitBsrMatrix<T>& m, int cap, const char* name) {
    Out out;
    static_cast<TileCodeValueCodec<Bits, T>&>(out) = build_exact_tile_code_value_codec<Bits>(m, cap, name);
    return out;
}
}  // namespace codec_detail

template <typename T>
Dict2Tile32ValueCodec<T> build_dict2_tile32_value_codec(const BitBsrMatrix<T>& m) {
    return codec_detail::named_tile_codec<Dict2Tile32ValueCodec<T>, 1>(m, 2, "dict2_tile32");
}
template <typename T>
Unique4Tile64ValueCodec<T> build_unique4_tile64_value_codec(const BitBsrMatrix<T>& m) {
    return codec_detail::named_tile_codec<Unique4Tile64ValueCodec<T>, 2>(m, 4, "unique4_tile64");
}
template <typename T>
Unique16Tile128ValueCodec<T> build_unique16_tile128_value_codec(const BitBsrMatrix<T>& m) {
    return codec_detail::named_tile_codec<Unique16Tile128ValueCodec<T>, 4>(m, 16, "unique16_tile128");
}
template <typename T>
Dict256Tile256ValueCodec<T> build_dict256_tile256_value_codec(const BitBsrMatrix<T>& m) {
    return codec_detail::named_tile_codec<Dict256Tile256ValueCodec<T>, 8>(m, 256, "dict256_tile256");
}
template <typename T>
Dict65536Tile512ValueCodec<T> build_dict65536_tile512_value_codec(const BitBsrMatrix<T>& m) {
    return codec_detail::named_tile_codec<Dict65536Tile512ValueCodec<T>, 16>(m, 65536, "dict65536_tile512");
}

// ---- 16-bit values -----------------------------------------------------------------

struct Round16NnzValueCodec {
    std::vector<std::uint16_t> values16;
    std::size_t payload_bytes() const { return values16.size() * 2; }
};

struct Round16Tile512ValueCodec {
    std::vector<std::uint32_t> tile_code_words;
    std::size_t payload_bytes() const { return tile_code_words.size() * 4; }
};

// encode_bits(value) -> 16 bits (float_to_bf16_bits / float_to_fp16_bits), per nnz
template <typename T, typename EncodeBitsFn>
Round16NnzValueCodec build_round16_nnz_value_codec(const BitBsrMatrix<T>& bitbsr, EncodeBitsFn encode_bits) {
    bitbsr.validate();
    Round16NnzValueCodec c;
    c.values16.reserve(bitbsr.values.size());
    for (const T v : bitbsr.values) c.values16.push_back(static_cast<std::uint16_t>(encode_bits(v)));
    return c;
}

// the same 16 bits per cell, two cells per word, 16 words per block
template <typename T, typename EncodeBitsFn>
Round16Tile512ValueCodec build_round16_tile512_value_codec(const BitBsrMatrix<T>& bitbsr, EncodeBitsFn encode_bits) {
    bitbsr.validate();
    Round16Tile512ValueCodec c;
    c.tile_code_words.assign(static_cast<size_t>(bitbsr.num_blocks()) * 16, 0);
    codec_detail::for_each_cell(bitbsr, [&](Offset b, int bit, Offset k) {
        const std::uint32_t v = static_cast<std::uint16_t>(encode_bits(bitbsr.values[k]));
        c.tile_code_words[static_cast<size_t>(b) * 16 + bit / 2] |= v << ((bit % 2) * 16);
    });
    return c;
}

// ---- block floating point --------------------------------------------------------

struct Bfp8BlkScaleValueCodec {
    std::vector<signed char> int8_values;
    std::vector<std::uint16_t> block_scale_bf16;
    std::size_t payload_bytes() const { return int8_values.size() + block_scale_bf16.size() * 2; }
};

struct Bfp4BlkScaleValueCodec {
    Offset nnz = 0;
    std::vector<std::uint8_t> packed_int4;
    std::vector<std::uint16_t> block_scale_bf16;
    std::size_t payload_bytes() const { return packed_int4.size() + block_scale_bf16.size() * 2; }
};

namespace codec_detail {
// Per block: scale = bf16(float(max|v| / qmax)) (1 when the block is all
// zero), q = clamp(lround(v / scale), -qmax, qmax); emit(k, q) per value.
template <typename T, typename Emit>
void block_quantize(const BitBsrMatrix<T>& m, double qmax, std::vector<std::uint16_t>& scales, Emit&& emit) {
    scales.assign(static_cast<size_t>(m.num_blocks()), 0);
    for (Offset b = 0; b < m.num_blocks(); ++b) {
        double mx = 0.0;
        for (Offset k = m.block_val_ptr[b]; k < m.block_val_ptr[b + 1]; ++k)
            mx = std::max(mx, std::abs(static_cast<double>(m.values[k])));
        float s = static_cast<float>(mx / qmax);
        if (s == 0.0f) s = 1.0f;
        scales[b] = float_to_bf16_bits(s);
        const double d = static_cast<double>(bf16_bits_to_float(scales[b]));
        const long lim = static_cast<long>(qmax);
        for (Offset k = m.block_val_ptr[b]; k < m.block_val_ptr[b + 1]; ++k)
            emit(k, std::max(-lim, std::min(lim, std::lround(static_cast<double>(m.values[k]) / d))));
    }
}
}  // namespace codec_detail

template <typename T>
Bfp8BlkScaleValueCodec build_bfp8_blkscale_value_codec(const BitBsrMatrix<T>& bitbsr) {
    bitbsr.validate();
    Bfp8BlkScaleValueCodec c;
    c.int8_values.assign(bitbsr.values.size(), 0);
    codec_detail::block_quantize(bitbsr, 127.0, c.block_scale_bf16,
                                 [&](Offset k, long q) { c.int8_values[k] = static_cast<signed char>(q); });
    return c;
}

// two signed 4-bit mantissas per byte: even nnz position in the low nibble
template <typename T>
Bfp4BlkScaleValueCodec build_bfp4_blkscale_value_codec(const BitBsrMatrix<T>& bitbsr) {
    bitbsr.validate();
    Bfp4BlkScaleValueCodec c;
    c.nnz = bitbsr.nnz();
    c.packed_int4.assign(static_cast<size_t>((bitbsr.nnz() + 1) / 2), 0);
    codec_detail::block_quantize(bitbsr, 7.0, c.block_scale_bf16, [&](Offset k, long q) {
        const std::uint8_t nib = static_cast<std::uint8_t>(q & 0xF);
        std::uint8_t& byte = c.packed_int4[static_cast<size_t>(k >> 1)];
        byte = (k & 1) ? static_cast<std::uint8_t>((byte & 0x0F) | (nib << 4))
                       : static_cast<std::uint8_t>((byte & 0xF0) | nib);
    });
    return c;
}

// ---- BFP8 with global outliers (gpu_value_codecs.cuh:319-461) -------------------
// The largest fraction of |values| (above the (1 - fraction) order statistic)
// leave the int8 stream (their slot is 0) for an exact side list of
// (row, col, value) in block-row / block / bit order; block scales cover the
// remaining values only.

template <typename T>
struct Bfp8OutlierBlkScaleValueCodec {
    Offset nnz = 0;
    Offset num_blocks = 0;
    Offset num_outliers = 0;
    std::vector<signed char> int8_values;
    std::vector<std::uint16_t> block_scale_bf16;
    std::vector<std::int32_t> outlier_rows;
    std::vector<std::int32_t> outlier_cols;
    std::vector<T> outlier_vals;
    std::size_t payload_bytes() const {
        return int8_values.size() + block_scale_bf16.size() * 2 +
               static_cast<std::size_t>(num_outliers) * (8 + sizeof(T));
    }
    // positions come from the bitmap: only the exact values are extra
    std::size_t value_only_payload_bytes() const {
        return int8_values.size() + block_scale_bf16.size() * 2 + static_cast<std::size_t>(num_outliers) * sizeof(T);
    }
};

template <typename T>
Bfp8OutlierBlkScaleValueCodec<T> build_bfp8_outlier_blkscale_value_codec(const BitBsrMatrix<T>& bitbsr,
                                                                         double outlier_fraction = 0.005) {
    bitbsr.validate();
    Bfp8OutlierBlkScaleValueCodec<T> c;
    const Offset nnz = bitbsr.nnz();
    c.nnz = nnz;
    c.num_blocks = bitbsr.num_blocks();
    c.int8_values.assign(static_cast<size_t>(nnz), 0);
    c.block_scale_bf16.assign(static_cast<size_t>(c.num_blocks), 0);
    std::vector<char> outlier(static_cast<size_t>(nnz), 0);
    if (outlier_fraction > 0.0 && nnz > 0) {
        std::vector<double> mag(static_cast<size_t>(nnz));
        for (Offset k = 0; k < nnz; ++k) mag[static_cast<size_t>(k)] = std::abs(static_cast<double>(bitbsr.values[k]));
        size_t at = static_cast<size_t>((1.0 - outlier_fraction) * static_cast<double>(nnz));
        if (at >= mag.size()) at = mag.size() - 1;
        std::vector<double> order(mag);
        std::nth_element(order.begin(), order.begin() + static_cast<std::ptrdiff_t>(at), order.end());
        const double threshold = order[at];
        for (size_t k = 0; k < mag.size(); ++k) outlier[k] = mag[k] > threshold ? 1 : 0;
    }
    for (Offset b = 0; b < c.num_blocks; ++b) {
        const Offset v0 = bitbsr.block_val_ptr[b], v1 = bitbsr.block_val_ptr[b + 1];
        double top = 0.0;
        for (Offset k = v0; k < v1; ++k)
            if (!outlier[static_cast<size_t>(k)]) top = std::max(top, std::abs(static_cast<double>(bitbsr.values[k])));
        float scale = static_cast<float>(top / 127.0);
        if (scale == 0.0f) scale = 1.0f;
        c.block_scale_bf16[static_cast<size_t>(b)] = float_to_bf16_bits(scale);
        const double step = static_cast<double>(bf16_bits_to_float(c.block_scale_bf16[static_cast<size_t>(b)]));
        for (Offset k = v0; k < v1; ++k) {
            if (outlier[static_cast<size_t>(k)]) continue;  // slot stays 0
            const long q = std::lround(static_cast<double>(bitbsr.values[k]) / step);
            c.int8_values[static_cast<size_t>(k)] = static_cast<signed char>(std::max(-127L, std::min(127L, q)));
        }
    }
    for (Index br = 0; br < bitbsr.num_block_rows; ++br)
        for (Offset b = bitbsr.block_row_ptr[br]; b < bitbsr.block_row_ptr[br + 1]; ++b) {
            const auto bm = static_cast<std::uint32_t>(bitbsr.bitmap_words[b]);
            for (int bit = 0; bit < 32; ++bit) {
                if (!(bm & (1u << bit))) continue;
                const Offset k = bitbsr.block_val_ptr[b] + popcount_word(bm & ((1u << bit) - 1u));
                if (!outlier[static_cast<size_t>(k)]) continue;
                c.outlier_rows.push_back(static_cast<std::int32_t>(br * bitbsr.block_rows + bit / bitbsr.block_cols));
                c.outlier_cols.push_back(
                    static_cast<std::int32_t>(bitbsr.block_col_idx[b] * bitbsr.block_cols + bit % bitbsr.block_cols));
                c.outlier_vals.push_back(bitbsr.values[static_cast<size_t>(k)]);
            }
        }
    c.num_outliers = static_cast<Offset>(c.outlier_vals.size());
    return c;
}


template <typename T>
struct K256Tile256BuildResult {
    TileCodeValueCodec<8, T> tile;
    int used_codebook_size = 0;
};

template <typename T>
struct LogKmeansTile256BuildResult {
    TileCodeValueCodec<8, T> tile;
    int used_codebook_size = 0;
};

// 8-bit codes into a 256-slot codebook (unused slots zero): the distinct
// values themselves when there are at most 256, else 256 k-means centres.
template <typename T>
K256Tile256BuildResult<T> build_k256_tile256_build_result(const BitBsrMatrix<T>& bitbsr) {
    constexpr int kSlots = 256;
    K256Tile256BuildResult<T> out;
    const std::vector<T>& vals = bitbsr.values;
    out.tile.codebook.assign(kSlots, T(0));
    out.tile.value_ids.assign(vals.size(), 0);
    out.tile.exact = false;
    if (!vals.empty()) {
        std::vector<double> sample;
        sample.reserve(vals.size());
        for (const T raw : vals) {
            if (!std::isfinite(static_cast<double>(raw)))
                throw std::runtime_error("K256 uint8 value codebook requires finite values");
            sample.push_back(static_cast<double>(raw));
        }
        const auto u = sorted_unique_values(vals, kSlots);
        if (static_cast<int>(u.size()) <= kSlots) {
            out.tile.exact = true;
            out.used_codebook_size = static_cast<int>(u.size());
            std::copy(u.begin(), u.end(), out.tile.codebook.begin());
            for (size_t i = 0; i < vals.size(); ++i)
                out.tile.value_ids[i] =
                    static_cast<std::uint32_t>(std::lower_bound(u.begin(), u.end(), vals[i]) - u.begin());
        } else {
            const auto centers = codec_detail::binned_kmeans_1d(std::move(sample), kSlots, 4096, 16);
            out.used_codebook_size = static_cast<int>(centers.size());
            for (size_t i = 0; i < centers.size(); ++i) out.tile.codebook[i] = static_cast<T>(centers[i]);
            for (size_t i = 0; i < vals.size(); ++i)
                out.tile.value_ids[i] =
                    static_cast<std::uint32_t>(codec_detail::nearest_center(centers, static_cast<double>(vals[i])));
        }
    }
    out.tile.tile_code_words = build_tile_code_words_from_value_ids<8>(bitbsr, out.tile.value_ids);
    return out;
}

// 8-bit codes over signed magnitudes: k-means of log2|v| (k <= 128 centres),
// codebook {-2^c, +2^c} per centre, code = 2 * centre + (v >= 0).
template <typename T>
LogKmeansTile256BuildResult<T> build_logkmeans_tile256_build_result(const BitBsrMatrix<T>& bitbsr, int requested_k,
                                                                    int histogram_bins = 4096,
                                                                    int iterations = 16) {
    bitbsr.validate();
    if (requested_k <= 0 || requested_k > 128)
        throw std::runtime_error("global_logkmeans value codec requires k in [1, 128]");
    std::vector<double> logs;
    logs.reserve(bitbsr.values.size());
    for (const T raw : bitbsr.values) {
        const double a = static_cast<double>(raw);
        if (!std::isfinite(a)) throw std::runtime_error("global_logkmeans value codec requires finite values");
        if (a == 0.0) throw std::runtime_error("global_logkmeans value codec requires nonzero BitBSR values");
        logs.push_back(std::log2(std::abs(a)));
    }
    const auto centers = codec_detail::binned_kmeans_1d(std::move(logs), requested_k, histogram_bins, iterations);
    if (centers.size() * 2 > 256) throw std::runtime_error("global_logkmeans value codec exceeded the uint8 codebook size");
    LogKmeansTile256BuildResult<T> out;
    for (const double c : centers) {
        const T m = static_cast<T>(std::exp2(c));
        out.tile.codebook.push_back(-m);
        out.tile.codebook.push_back(m);
    }
    out.used_codebook_size = static_cast<int>(out.tile.codebook.size());
    out.tile.exact = false;
    out.tile.value_ids.resize(bitbsr.values.size());
    for (size_t i = 0; i < bitbsr.values.size(); ++i) {
        const double a = static_cast<double>(bitbsr.values[i]);
        const int j = codec_detail::nearest_center(centers, std::log2(std::abs(a)));
        out.tile.value_ids[i] = static_cast<std::uint32_t>(j * 2 + (a < 0.0 ? 0 : 1));
    }
    out.tile.tile_code_words = build_tile_code_words_from_value_ids<8>(bitbsr, out.tile.value_ids);
    return out;
}

// ---- checked builders (gpu_value_codecs.cuh:760-875): the 8x4 tile shape first --

template <typename T>
void validate_tile_shape_8x4(const BitBsrMatrix<T>& bitbsr) {
    if (bitbsr.block_rows != 8 || bitbsr.block_cols != 4 || bitbsr.words_per_block != 1)
        throw std::runtime_error("tile value codecs require 8x4 BitBSR blocks");
}

template <typename T>
std::vector<std::uint32_t> build_checked_sign2_tile32_masks(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_sign2_tile32_masks(bitbsr);
}

template <typename T>
Round16NnzValueCodec build_checked_fp16_nnz_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_round16_nnz_value_codec(bitbsr, [](T v) { return float_to_fp16_bits(static_cast<float>(v)); });
}

template <typename T>
Round16NnzValueCodec build_checked_bf16_nnz_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_round16_nnz_value_codec(bitbsr, [](T v) { return float_to_bf16_bits(static_cast<float>(v)); });
}

template <typename T>
Bfp8BlkScaleValueCodec build_checked_bfp8_blkscale_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_bfp8_blkscale_value_codec(bitbsr);
}

template <typename T>
Bfp8OutlierBlkScaleValueCodec<T> build_checked_bfp8_outlier_blkscale_value_codec(const BitBsrMatrix<T>& bitbsr,
                                                                                 double outlier_fraction = 0.005) {
    validate_tile_shape_8x4(bitbsr);
    return build_bfp8_outlier_blkscale_value_codec(bitbsr, outlier_fraction);
}

template <typename T>
Bfp4BlkScaleValueCodec build_checked_bfp4_blkscale_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_bfp4_blkscale_value_codec(bitbsr);
}

template <typename T>
T build_checked_const_c_value(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_const_c_value(bitbsr);
}

template <typename T>
Sign2ScaleTile32ValueCodec<T> build_checked_sign2_scale_tile32_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_sign2_scale_tile32_value_codec(bitbsr);
}

template <typename T>
Dict2Tile32ValueCodec<T> build_checked_dict2_tile32_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_dict2_tile32_value_codec(bitbsr);
}

template <typename T>
Unique4Tile64ValueCodec<T> build_checked_unique4_tile64_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_unique4_tile64_value_codec(bitbsr);
}

template <typename T>
Unique16Tile128ValueCodec<T> build_checked_unique16_tile128_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_unique16_tile128_value_codec(bitbsr);
}

template <typename T>
Dict256Tile256ValueCodec<T> build_checked_dict256_tile256_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_dict256_tile256_value_codec(bitbsr);
}

template <typename T>
Dict65536Tile512ValueCodec<T> build_checked_dict65536_tile512_value_codec(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_dict65536_tile512_value_codec(bitbsr);
}

template <typename T>
K256Tile256BuildResult<T> build_checked_k256_tile256_build_result(const BitBsrMatrix<T>& bitbsr) {
    validate_tile_shape_8x4(bitbsr);
    return build_k256_tile256_build_result(bitbsr);
}

template <typename T>
LogKmeansTile256BuildResult<T> build_checked_logkmeans_tile256_build_result(const BitBsrMatrix<T>& bitbsr,
                                                                            int requested_k) {
    validate_tile_shape_8x4(bitbsr);
    return build_logkmeans_tile256_build_result(bitbsr, requested_k);
}

}  // namespace structural
