// types.hpp -- index and bitmap types of the structural:: API (int32 offsets,
// 32-bit block bitmap), as in structural/include/structural/types.hpp:7-11.
#pragma once

#include <cstdint>

namespace structural {

using Index = std::int32_t;
using Offset = std::int32_t;
using BitmapWord = std::uint32_t;

constexpr int kBitmapWordBits = static_cast<int>(sizeof(BitmapWord) * 8);

}  // namespace structural
