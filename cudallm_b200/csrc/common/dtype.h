// Tensor and weight type codes of the .cudallm format (wasiqnauman/cudallm src/common/dtype.h:7-8,
// python/cudallm/format.py:10-20). The numeric values are part of the on-disk format.
#pragma once

#include <cstdint>

namespace cudallm {

enum class DType : uint32_t { F32 = 0, BF16 = 1, F16 = 2, I8 = 3, I4X2 = 4 };
enum class WeightType : uint32_t { BF16 = 1, INT8 = 3, INT4 = 4 };
enum class KvType : int { F16 = 0, BF16 = 1 };

inline const char* to_string(WeightType w) {
    switch (w) {
        case WeightType::BF16: return "bf16";
        case WeightType::INT8: return "int8";
        case WeightType::INT4: return "int4";
    }
    return "unknown";
}

// Bytes of one stored weight row of `cols` columns.
inline uint64_t row_bytes(WeightType w, uint64_t cols) {
    switch (w) {
        case WeightType::BF16: return cols * 2;
        case WeightType::INT8: return cols;
        case WeightType::INT4: return cols / 2;
    }
    return 0;
}

}  // namespace cudallm
