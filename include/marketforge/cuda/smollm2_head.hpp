// The output-head tail of CudaSmolLm2::forward on the B200 head (no
// reference counterpart as a class: it replaces the tail of
// src/cuda/smollm2.cu:459-501, everything after the decoder layers).
//
// The reference's tail copies the last row of the decoder output into
// last_hidden_, runs rms_norm_f16 into last_normalized_, then either
// linear_f16 (cuBLAS fp16 logits [1, V]) + greedy_select_f16, or — for
// restricted decode — restricted_output_head_f16 over a padded table of at
// most 128 ids copied from the host every token
// (include/marketforge/cuda/smollm2.hpp:33), and finally copies the token to
// the host and synchronises.  SmolLm2OutputHead does the same job with one
// kernel per token and no cap:
//   * select_restricted: the final RMSNorm fused into the ragged head over
//     any number of allowed ids already on the device;
//   * select_grammar: the final RMSNorm fused into the device grammar step
//     (allowed-set lookup, head, advance of the device-resident state), so
//     no allowed ids cross PCIe at all;
//   * select_greedy: the full-vocabulary swap for linear_f16 +
//     greedy_select_f16 — the fused norm + head over every vocabulary id,
//     FP32 scores, no logits written (the reference rounds logits to fp16,
//     which can flip near-ties).
// Each reads the decoder output's last row in place (no copy), copies the
// selected token to the host and synchronises the stream, as forward()
// does, and returns it.  Tie and NaN rules are greedy.hpp's.
#pragma once

#include <cstdint>

#include "marketforge/core/result.hpp"
#include "marketforge/core/status.hpp"
#include "marketforge/cuda/cuda_stream.hpp"
#include "marketforge/cuda/device_buffer.hpp"

namespace marketforge::cuda {

struct SmolLm2OutputHeadSpec {
  std::uint64_t hidden_size{576};
  std::uint64_t vocabulary_size{49'152};
  float rms_norm_epsilon{1.0e-5F};
};

class SmolLm2OutputHead {
public:
  // Allocates the head's device state once (workspace, CSR offsets, the
  // all-vocabulary id list, the selected-token slot).
  [[nodiscard]] static Result<SmolLm2OutputHead> create(SmolLm2OutputHeadSpec spec,
                                                        StreamHandle stream) noexcept;

  SmolLm2OutputHead(SmolLm2OutputHead&&) noexcept = default;
  SmolLm2OutputHead& operator=(SmolLm2OutputHead&&) noexcept = default;
  SmolLm2OutputHead(const SmolLm2OutputHead&) = delete;
  SmolLm2OutputHead& operator=(const SmolLm2OutputHead&) = delete;

  // hidden: the decoder's output, fp16 [rows, hidden_size]; its last row is
  // the one decoded.  final_norm: fp16 [hidden_size].  allowed_ids: int32 /
  // u32 device ids, allowed_count of them (any count >= 1).
  [[nodiscard]] Result<std::uint32_t> select_restricted(
      const DeviceBuffer& hidden, std::uint64_t rows, const DeviceBuffer& final_norm,
      const DeviceBuffer& embedding, const DeviceBuffer& allowed_ids,
      std::uint64_t allowed_count, StreamHandle stream) noexcept;

  // The grammar on the device (TokenDfa's CSR: state_offsets int32
  // [num_states + 1], arc_tokens / arc_next [arcs]); state: u32 [1], read
  // and advanced on the device.  A state with no arcs gives the sentinel
  // (restricted_greedy_invalid_token_id) and keeps the state.
  [[nodiscard]] Result<std::uint32_t> select_grammar(
      const DeviceBuffer& hidden, std::uint64_t rows, const DeviceBuffer& final_norm,
      const DeviceBuffer& embedding, const DeviceBuffer& state_offsets,
      const DeviceBuffer& arc_tokens, const DeviceBuffer& arc_next, DeviceBuffer& state,
      std::uint64_t num_states, StreamHandle stream) noexcept;

  // Full vocabulary (the swap for linear_f16 + greedy_select_f16).
  [[nodiscard]] Result<std::uint32_t> select_greedy(const DeviceBuffer& hidden,
                                                    std::uint64_t rows,
                                                    const DeviceBuffer& final_norm,
                                                    const DeviceBuffer& embedding,
                                                    StreamHandle stream) noexcept;

private:
  SmolLm2OutputHead() noexcept = default;
  [[nodiscard]] Result<std::uint32_t> finish(StreamHandle stream) noexcept;

  SmolLm2OutputHeadSpec spec_{};
  DeviceBuffer workspace_{};    // ragged-head / grammar workspace (one row)
  DeviceBuffer offsets_{};      // int32 [2]: 0, count of the current allowed set
  DeviceBuffer all_ids_{};      // int32 [V]: 0 .. V-1 (select_greedy's candidates)
  DeviceBuffer selected_{};     // u32 [1]
  DeviceBuffer next_state_{};   // u32 [1] (select_grammar's advanced state)
  std::int32_t host_offsets_[2]{0, 0};
  std::uint32_t host_selected_{0};
};

} // namespace marketforge::cuda
