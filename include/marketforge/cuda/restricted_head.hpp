// New batched entry points in the reference's style (no reference
// counterpart; they extend greedy.hpp): the ragged CSR head, the device DFA
// step / decode, and the dense full-vocabulary head over a vocabulary shard.
// Contracts are those of include/mf_head.h; workspaces are caller-owned
// DeviceBuffers, zero-filled once (RestrictedHeadWorkspace does that) and
// left zero by every call.
#pragma once

#include <cstdint>

#include "marketforge/core/result.hpp"
#include "marketforge/core/status.hpp"
#include "marketforge/cuda/cuda_stream.hpp"
#include "marketforge/cuda/device_buffer.hpp"

namespace marketforge::cuda {

// A zero-filled workspace for up to `rows` rows of the ragged, DFA or dense head.
[[nodiscard]] Result<DeviceBuffer> allocate_head_workspace(std::uint64_t rows,
                                                           StreamHandle stream) noexcept;

// Row r's candidates are ids[offsets[r] .. offsets[r+1]) (int32 CSR).
// token_ids: u32 [rows]; scores: f32 [rows] or an empty buffer.
[[nodiscard]] Status restricted_output_head_csr_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& embedding, const DeviceBuffer& offsets,
    const DeviceBuffer& ids, DeviceBuffer& token_ids, DeviceBuffer& scores,
    DeviceBuffer& workspace, std::uint64_t rows, std::uint64_t hidden_size,
    std::uint64_t vocabulary_size, StreamHandle stream) noexcept;

// Launch option of the overload below (MF_LAUNCH_OVERLAP_PREVIOUS): the call
// may overlap the tail of the previous kernel on `stream`, which must not
// write this call's inputs (consecutive calls on independent batches).
inline constexpr std::uint32_t launch_overlap_previous = 1u;
[[nodiscard]] Status restricted_output_head_csr_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& embedding, const DeviceBuffer& offsets,
    const DeviceBuffer& ids, DeviceBuffer& token_ids, DeviceBuffer& scores,
    DeviceBuffer& workspace, std::uint64_t rows, std::uint64_t hidden_size,
    std::uint64_t vocabulary_size, std::uint32_t launch_flags, StreamHandle stream) noexcept;

// The same with the final RMSNorm fused in front: hidden holds the last
// layer's un-normalised rows, gamma the norm weight fp16 [hidden_size]
// (replaces rms_norm_f16 + the head, src/cuda/smollm2.cu:474-492).
[[nodiscard]] Status restricted_output_head_csr_rmsnorm_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& gamma, float epsilon,
    const DeviceBuffer& embedding, const DeviceBuffer& offsets, const DeviceBuffer& ids,
    DeviceBuffer& token_ids, DeviceBuffer& scores, DeviceBuffer& workspace, std::uint64_t rows,
    std::uint64_t hidden_size, std::uint64_t vocabulary_size, StreamHandle stream) noexcept;

// `steps` device DFA steps (allowed-set lookup, head, advance; TokenDfa's
// CSR: state_offsets / arc_tokens / arc_next).  state_trace u32
// [steps + 1, batch] with row 0 = initial states; token_trace u32 [steps, batch].
[[nodiscard]] Status dfa_decode_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& embedding, const DeviceBuffer& state_offsets,
    const DeviceBuffer& arc_tokens, const DeviceBuffer& arc_next, DeviceBuffer& state_trace,
    DeviceBuffer& token_trace, DeviceBuffer& workspace, std::uint64_t steps, std::uint64_t batch,
    std::uint64_t num_states, std::uint64_t hidden_size, std::uint64_t vocabulary_size,
    StreamHandle stream) noexcept;

// Full-vocabulary greedy head over vocabulary ids [vocab_begin, vocab_begin +
// vocab_rows) (replaces linear_f16 + greedy_select_f16).  keys: u64 [rows]
// packed keys for a cross-shard max, or empty; token_ids: u32 [rows] or empty.
[[nodiscard]] Status dense_output_head_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& embedding, DeviceBuffer& keys,
    DeviceBuffer& token_ids, DeviceBuffer& workspace, std::uint64_t rows,
    std::uint64_t hidden_size, std::uint64_t vocab_rows, std::uint64_t vocab_begin,
    StreamHandle stream) noexcept;

// Vocabulary shards on several GPUs, merged inside the kernel
// (mf_dense_head_sharded_f16): one process per GPU; exchange[q] is rank q's
// exchange buffer (mf_exchange_alloc / mf_exchange_open_peer) as mapped in
// this process; every rank gets the global ids (and merged keys).
[[nodiscard]] Status dense_output_head_sharded_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& embedding, DeviceBuffer& keys,
    DeviceBuffer& token_ids, DeviceBuffer& workspace, std::uint64_t rows,
    std::uint64_t hidden_size, std::uint64_t vocab_rows, std::uint64_t vocab_begin,
    void* const* exchange, std::uint64_t exchange_bytes, std::uint32_t world, std::uint32_t rank,
    StreamHandle stream) noexcept;

}  // namespace marketforge::cuda
