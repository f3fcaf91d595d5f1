// marketforge::cuda greedy selection and the fused restricted head — the
// reference's interface (include/marketforge/cuda/greedy.hpp:9-51) with the
// same signatures and contracts, implemented by the B200 kernels behind
// include/mf_head.h.  Equal scores resolve to the lowest token id, NaN never
// wins, an all-NaN valid candidate set falls back to its lowest id, and bad
// device-side rows emit restricted_greedy_invalid_token_id.
#pragma once

#include <cstdint>

#include "marketforge/core/status.hpp"
#include "marketforge/cuda/cuda_stream.hpp"
#include "marketforge/cuda/device_buffer.hpp"

namespace marketforge::cuda {

inline constexpr std::uint32_t restricted_greedy_invalid_token_id = UINT32_MAX;

// greedy.hpp:17-21: argmax per row of fp16 logits[rows, vocabulary_size].
[[nodiscard]] Status greedy_select_f16(const DeviceBuffer& logits, DeviceBuffer& token_ids,
                                       std::uint64_t rows, std::uint64_t vocabulary_size,
                                       StreamHandle stream) noexcept;

// greedy.hpp:29-33: masked argmax over a padded [rows, maximum] candidate table.
[[nodiscard]] Status restricted_greedy_select_f16(
    const DeviceBuffer& logits, const DeviceBuffer& allowed_token_ids,
    const DeviceBuffer& allowed_token_counts, DeviceBuffer& token_ids, std::uint64_t rows,
    std::uint64_t vocabulary_size, std::uint64_t maximum_allowed_tokens,
    StreamHandle stream) noexcept;

// greedy.hpp:43-49: tied projection + restricted argmax, no full logits.
[[nodiscard]] Status restricted_output_head_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& embedding,
    const DeviceBuffer& allowed_token_ids, const DeviceBuffer& allowed_token_counts,
    DeviceBuffer& token_ids, std::uint64_t rows, std::uint64_t hidden_size,
    std::uint64_t vocabulary_size, std::uint64_t maximum_allowed_tokens,
    StreamHandle stream) noexcept;

}  // namespace marketforge::cuda
