// marketforge::cuda head functions over the C-ABI of include/mf_head.h.  Each
// passes the buffers' exact byte sizes through, so the reference's
// size/aliasing validation (src/cuda/greedy.cu:349-399) happens in one place.
#include <cuda_runtime_api.h>

#include "marketforge/cuda/greedy.hpp"
#include "marketforge/cuda/restricted_head.hpp"
#include "mf_head.h"

namespace marketforge::cuda {
namespace {

Status to_status(mf_status s) noexcept { return Status{static_cast<ErrorCode>(s.code), s.detail}; }
const void* ca(const DeviceBuffer& b) noexcept { return reinterpret_cast<const void*>(b.address().value); }
void* ma(DeviceBuffer& b) noexcept { return reinterpret_cast<void*>(b.address().value); }
void* st(StreamHandle h) noexcept { return reinterpret_cast<void*>(h.value); }

}  // namespace

Status greedy_select_f16(const DeviceBuffer& logits, DeviceBuffer& token_ids, std::uint64_t rows,
                         std::uint64_t vocabulary_size, StreamHandle stream) noexcept {
  return to_status(mf_greedy_select_f16(ca(logits), logits.size_bytes(), ma(token_ids),
                                        token_ids.size_bytes(), rows, vocabulary_size, st(stream)));
}

Status restricted_greedy_select_f16(const DeviceBuffer& logits, const DeviceBuffer& allowed,
                                    const DeviceBuffer& counts, DeviceBuffer& token_ids,
                                    std::uint64_t rows, std::uint64_t vocabulary_size,
                                    std::uint64_t maximum, StreamHandle stream) noexcept {
  return to_status(mf_restricted_greedy_select_f16(
      ca(logits), logits.size_bytes(), ca(allowed), allowed.size_bytes(), ca(counts),
      counts.size_bytes(), ma(token_ids), token_ids.size_bytes(), rows, vocabulary_size, maximum,
      st(stream)));
}

Status restricted_output_head_f16(const DeviceBuffer& hidden, const DeviceBuffer& embedding,
                                  const DeviceBuffer& allowed, const DeviceBuffer& counts,
                                  DeviceBuffer& token_ids, std::uint64_t rows,
                                  std::uint64_t hidden_size, std::uint64_t vocabulary_size,
                                  std::uint64_t maximum, StreamHandle stream) noexcept {
  return to_status(mf_restricted_output_head_f16(
      ca(hidden), hidden.size_bytes(), ca(embedding), embedding.size_bytes(), ca(allowed),
      allowed.size_bytes(), ca(counts), counts.size_bytes(), ma(token_ids),
      token_ids.size_bytes(), rows, hidden_size, vocabulary_size, maximum, st(stream)));
}

Result<DeviceBuffer> allocate_head_workspace(std::uint64_t rows, StreamHandle stream) noexcept {
  std::uint64_t bytes = mf_head_workspace_bytes(rows);
  if (mf_dense_workspace_bytes(rows) > bytes) bytes = mf_dense_workspace_bytes(rows);
  if (mf_dfa_workspace_bytes(rows) > bytes) bytes = mf_dfa_workspace_bytes(rows);
  auto buf = DeviceBuffer::allocate(bytes);
  if (!buf) return buf;
  const auto e = cudaMemsetAsync(reinterpret_cast<void*>(buf.value().address().value), 0,
                                 (size_t)bytes, reinterpret_cast<cudaStream_t>(stream.value));
  if (e != cudaSuccess)
    return Result<DeviceBuffer>::failure(
        Status::failure(ErrorCode::cuda_runtime_failure, (std::uint32_t)e));
  return buf;
}

Status restricted_output_head_csr_f16(const DeviceBuffer& hidden, const DeviceBuffer& embedding,
                                      const DeviceBuffer& offsets, const DeviceBuffer& ids,
                                      DeviceBuffer& token_ids, DeviceBuffer& scores,
                                      DeviceBuffer& workspace, std::uint64_t rows,
                                      std::uint64_t hidden_size, std::uint64_t vocabulary_size,
                                      StreamHandle stream) noexcept {
  return to_status(mf_head_restricted_csr_f16(
      ca(hidden), hidden.size_bytes(), ca(embedding), embedding.size_bytes(), ca(offsets),
      offsets.size_bytes(), ca(ids), ids.size_bytes(), ma(token_ids), token_ids.size_bytes(),
      scores.address().valid() ? ma(scores) : nullptr, scores.size_bytes(), ma(workspace),
      workspace.size_bytes(), rows, hidden_size, vocabulary_size, st(stream)));
}

Status restricted_output_head_csr_rmsnorm_f16(
    const DeviceBuffer& hidden, const DeviceBuffer& gamma, float epsilon,
    const DeviceBuffer& embedding, const DeviceBuffer& offsets, const DeviceBuffer& ids,
    DeviceBuffer& token_ids, DeviceBuffer& scores, DeviceBuffer& workspace, std::uint64_t rows,
    std::uint64_t hidden_size, std::uint64_t vocabulary_size, StreamHandle stream) noexcept {
  return to_status(mf_head_restricted_csr_rmsnorm_f16(
      ca(hidden), hidden.size_bytes(), ca(gamma), gamma.size_bytes(), epsilon, ca(embedding),
      embedding.size_bytes(), ca(offsets), offsets.size_bytes(), ca(ids), ids.size_bytes(),
      ma(token_ids), token_ids.size_bytes(), scores.address().valid() ? ma(scores) : nullptr,
      scores.size_bytes(), ma(workspace), workspace.size_bytes(), rows, hidden_size,
      vocabulary_size, st(stream)));
}

Status dfa_decode_f16(const DeviceBuffer& hidden, const DeviceBuffer& embedding,
                      const DeviceBuffer& state_offsets, const DeviceBuffer& arc_tokens,
                      const DeviceBuffer& arc_next, DeviceBuffer& state_trace,
                      DeviceBuffer& token_trace, DeviceBuffer& workspace, std::uint64_t steps,
                      std::uint64_t batch, std::uint64_t num_states, std::uint64_t hidden_size,
                      std::uint64_t vocabulary_size, StreamHandle stream) noexcept {
  return to_status(mf_dfa_decode_f16(
      ca(hidden), hidden.size_bytes(), ca(embedding), embedding.size_bytes(), ca(state_offsets),
      state_offsets.size_bytes(), ca(arc_tokens), arc_tokens.size_bytes(), ca(arc_next),
      arc_next.size_bytes(), ma(state_trace), state_trace.size_bytes(), ma(token_trace),
      token_trace.size_bytes(), nullptr, 0, ma(workspace), workspace.size_bytes(), steps, batch,
      num_states, hidden_size, vocabulary_size, st(stream)));
}

Status dense_output_head_f16(const DeviceBuffer& hidden, const DeviceBuffer& embedding,
                             DeviceBuffer& keys, DeviceBuffer& token_ids, DeviceBuffer& workspace,
                             std::uint64_t rows, std::uint64_t hidden_size,
                             std::uint64_t vocab_rows, std::uint64_t vocab_begin,
                             StreamHandle stream) noexcept {
  return to_status(mf_dense_head_f16(
      ca(hidden), hidden.size_bytes(), ca(embedding), embedding.size_bytes(),
      keys.address().valid() ? ma(keys) : nullptr, keys.size_bytes(),
      token_ids.address().valid() ? ma(token_ids) : nullptr, token_ids.size_bytes(), nullptr, 0,
      ma(workspace), workspace.size_bytes(), rows, hidden_size, vocab_rows, vocab_begin,
      st(stream)));
}

Status restricted_output_head_csr_f16(const DeviceBuffer& hidden, const DeviceBuffer& embedding,
                                      const DeviceBuffer& offsets, const DeviceBuffer& ids,
                                      DeviceBuffer& token_ids, DeviceBuffer& scores,
                                      DeviceBuffer& workspace, std::uint64_t rows,
                                      std::uint64_t hidden_size, std::uint64_t vocabulary_size,
                                      std::uint32_t launch_flags, StreamHandle stream) noexcept {
  return to_status(mf_head_restricted_csr_f16_ex(
      ca(hidden), hidden.size_bytes(), ca(embedding), embedding.size_bytes(), ca(offsets),
      offsets.size_bytes(), ids.address().valid() ? ca(ids) : nullptr, ids.size_bytes(),
      ma(token_ids), token_ids.size_bytes(), scores.address().valid() ? ma(scores) : nullptr,
      scores.size_bytes(), ma(workspace), workspace.size_bytes(), rows, hidden_size,
      vocabulary_size, launch_flags, st(stream)));
}

Status dense_output_head_sharded_f16(const DeviceBuffer& hidden, const DeviceBuffer& embedding,
                                     DeviceBuffer& keys, DeviceBuffer& token_ids,
                                     DeviceBuffer& workspace, std::uint64_t rows,
                                     std::uint64_t hidden_size, std::uint64_t vocab_rows,
                                     std::uint64_t vocab_begin, void* const* exchange,
                                     std::uint64_t exchange_bytes, std::uint32_t world,
                                     std::uint32_t rank, StreamHandle stream) noexcept {
  return to_status(mf_dense_head_sharded_f16(
      ca(hidden), hidden.size_bytes(), ca(embedding), embedding.size_bytes(),
      keys.address().valid() ? ma(keys) : nullptr, keys.size_bytes(),
      token_ids.address().valid() ? ma(token_ids) : nullptr, token_ids.size_bytes(), nullptr, 0,
      ma(workspace), workspace.size_bytes(), rows, hidden_size, vocab_rows, vocab_begin, exchange,
      exchange_bytes, world, rank, 0u, st(stream)));
}

}  // namespace marketforge::cuda
