// SmolLm2OutputHead: the tail of CudaSmolLm2::forward
// (src/cuda/smollm2.cu:459-501) over the C-ABI of include/mf_head.h.
#include "marketforge/cuda/smollm2_head.hpp"

#include <cstddef>
#include <utility>
#include <vector>

#include <cuda_runtime_api.h>

#include "marketforge/cuda/greedy.hpp"
#include "mf_head.h"

namespace marketforge::cuda {
namespace {

Status to_status(mf_status s) noexcept { return Status{static_cast<ErrorCode>(s.code), s.detail}; }
Status runtime(cudaError_t e) noexcept {
  return e == cudaSuccess ? Status::success()
                          : Status::failure(ErrorCode::cuda_runtime_failure,
                                            static_cast<std::uint32_t>(e));
}
const char* cb(const DeviceBuffer& b) noexcept {
  return reinterpret_cast<const char*>(b.address().value);
}
void* mb(DeviceBuffer& b) noexcept { return reinterpret_cast<void*>(b.address().value); }
cudaStream_t cs(StreamHandle h) noexcept { return reinterpret_cast<cudaStream_t>(h.value); }
void* vs(StreamHandle h) noexcept { return reinterpret_cast<void*>(h.value); }

template <typename T>
Result<T> fail(Status s) noexcept {
  return Result<T>::failure(s);
}

// The decoder output's last row: hidden [rows, hidden_size] fp16, read in
// place (the reference copies it into last_hidden_ first).
Status last_row(const DeviceBuffer& hidden, std::uint64_t rows, std::uint64_t hidden_size,
                const char** row) noexcept {
  if (rows == 0 || hidden_size == 0 || !hidden.address().valid() ||
      hidden.size_bytes() != rows * hidden_size * 2)
    return Status::failure(ErrorCode::invalid_argument);
  *row = cb(hidden) + (rows - 1) * hidden_size * 2;
  return Status::success();
}

}  // namespace

Result<SmolLm2OutputHead> SmolLm2OutputHead::create(SmolLm2OutputHeadSpec spec,
                                                    StreamHandle stream) noexcept {
  if (spec.hidden_size == 0 || spec.vocabulary_size == 0 || !stream.valid() ||
      !(spec.rms_norm_epsilon > 0.0F))
    return fail<SmolLm2OutputHead>(Status::failure(ErrorCode::invalid_argument));
  if (spec.vocabulary_size > static_cast<std::uint64_t>(INT32_MAX))
    return fail<SmolLm2OutputHead>(Status::failure(ErrorCode::resource_limit));
  SmolLm2OutputHead h;
  h.spec_ = spec;
  const std::uint64_t ws = mf_head_workspace_bytes(1) > mf_dfa_workspace_bytes(1)
                               ? mf_head_workspace_bytes(1)
                               : mf_dfa_workspace_bytes(1);
  auto w = DeviceBuffer::allocate(ws);
  auto o = DeviceBuffer::allocate(2 * sizeof(std::int32_t));
  auto a = DeviceBuffer::allocate(spec.vocabulary_size * sizeof(std::int32_t));
  auto s = DeviceBuffer::allocate(sizeof(std::uint32_t));
  auto n = DeviceBuffer::allocate(sizeof(std::uint32_t));
  if (!w) return fail<SmolLm2OutputHead>(w.status());
  if (!o) return fail<SmolLm2OutputHead>(o.status());
  if (!a) return fail<SmolLm2OutputHead>(a.status());
  if (!s) return fail<SmolLm2OutputHead>(s.status());
  if (!n) return fail<SmolLm2OutputHead>(n.status());
  h.workspace_ = std::move(w).value();
  h.offsets_ = std::move(o).value();
  h.all_ids_ = std::move(a).value();
  h.selected_ = std::move(s).value();
  h.next_state_ = std::move(n).value();
  std::vector<std::int32_t> ids(spec.vocabulary_size);
  for (std::size_t i = 0; i < ids.size(); ++i) ids[i] = static_cast<std::int32_t>(i);
  Status st = runtime(cudaMemsetAsync(mb(h.workspace_), 0, ws, cs(stream)));
  if (st.ok())
    st = runtime(cudaMemcpyAsync(mb(h.all_ids_), ids.data(), ids.size() * sizeof(std::int32_t),
                                 cudaMemcpyHostToDevice, cs(stream)));
  if (st.ok()) st = runtime(cudaStreamSynchronize(cs(stream)));  // `ids` is a local
  if (!st.ok()) return fail<SmolLm2OutputHead>(st);
  return Result<SmolLm2OutputHead>::success(std::move(h));
}

Result<std::uint32_t> SmolLm2OutputHead::finish(StreamHandle stream) noexcept {
  Status st = runtime(cudaMemcpyAsync(&host_selected_, mb(selected_), sizeof(host_selected_),
                                      cudaMemcpyDeviceToHost, cs(stream)));
  if (st.ok()) st = runtime(cudaStreamSynchronize(cs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  return Result<std::uint32_t>::success(host_selected_);
}

Result<std::uint32_t> SmolLm2OutputHead::select_restricted(
    const DeviceBuffer& hidden, std::uint64_t rows, const DeviceBuffer& final_norm,
    const DeviceBuffer& embedding, const DeviceBuffer& allowed_ids, std::uint64_t allowed_count,
    StreamHandle stream) noexcept {
  const char* row = nullptr;
  Status st = last_row(hidden, rows, spec_.hidden_size, &row);
  if (!st.ok()) return fail<std::uint32_t>(st);
  if (allowed_count == 0 || !stream.valid() ||
      allowed_ids.size_bytes() < allowed_count * sizeof(std::int32_t))
    return fail<std::uint32_t>(Status::failure(ErrorCode::invalid_argument));
  if (allowed_count > static_cast<std::uint64_t>(INT32_MAX))
    return fail<std::uint32_t>(Status::failure(ErrorCode::resource_limit));
  host_offsets_[0] = 0;
  host_offsets_[1] = static_cast<std::int32_t>(allowed_count);
  st = runtime(cudaMemcpyAsync(mb(offsets_), host_offsets_, sizeof(host_offsets_),
                               cudaMemcpyHostToDevice, cs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  st = to_status(mf_head_restricted_csr_rmsnorm_f16(
      row, spec_.hidden_size * 2, cb(final_norm), final_norm.size_bytes(),
      spec_.rms_norm_epsilon, cb(embedding), embedding.size_bytes(), cb(offsets_),
      offsets_.size_bytes(), cb(allowed_ids), allowed_count * sizeof(std::int32_t), mb(selected_),
      selected_.size_bytes(), nullptr, 0, mb(workspace_), workspace_.size_bytes(), 1,
      spec_.hidden_size, spec_.vocabulary_size, vs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  return finish(stream);
}

Result<std::uint32_t> SmolLm2OutputHead::select_grammar(
    const DeviceBuffer& hidden, std::uint64_t rows, const DeviceBuffer& final_norm,
    const DeviceBuffer& embedding, const DeviceBuffer& state_offsets,
    const DeviceBuffer& arc_tokens, const DeviceBuffer& arc_next, DeviceBuffer& state,
    std::uint64_t num_states, StreamHandle stream) noexcept {
  const char* row = nullptr;
  Status st = last_row(hidden, rows, spec_.hidden_size, &row);
  if (!st.ok()) return fail<std::uint32_t>(st);
  if (state.size_bytes() != sizeof(std::uint32_t))
    return fail<std::uint32_t>(Status::failure(ErrorCode::invalid_argument));
  st = to_status(mf_dfa_head_step_rmsnorm_f16(
      row, spec_.hidden_size * 2, cb(final_norm), final_norm.size_bytes(),
      spec_.rms_norm_epsilon, cb(embedding), embedding.size_bytes(), cb(state_offsets),
      state_offsets.size_bytes(), cb(arc_tokens), arc_tokens.size_bytes(), cb(arc_next),
      arc_next.size_bytes(), cb(state), state.size_bytes(), mb(next_state_),
      next_state_.size_bytes(), mb(selected_), selected_.size_bytes(), nullptr, 0,
      mb(workspace_), workspace_.size_bytes(), 1, num_states, spec_.hidden_size,
      spec_.vocabulary_size, vs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  st = runtime(cudaMemcpyAsync(mb(state), cb(next_state_), sizeof(std::uint32_t),
                               cudaMemcpyDeviceToDevice, cs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  return finish(stream);
}

Result<std::uint32_t> SmolLm2OutputHead::select_greedy(const DeviceBuffer& hidden,
                                                       std::uint64_t rows,
                                                       const DeviceBuffer& final_norm,
                                                       const DeviceBuffer& embedding,
                                                       StreamHandle stream) noexcept {
  const char* row = nullptr;
  Status st = last_row(hidden, rows, spec_.hidden_size, &row);
  if (!st.ok()) return fail<std::uint32_t>(st);
  if (!stream.valid()) return fail<std::uint32_t>(Status::failure(ErrorCode::invalid_argument));
  host_offsets_[0] = 0;
  host_offsets_[1] = static_cast<std::int32_t>(spec_.vocabulary_size);
  st = runtime(cudaMemcpyAsync(mb(offsets_), host_offsets_, sizeof(host_offsets_),
                               cudaMemcpyHostToDevice, cs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  st = to_status(mf_head_restricted_csr_rmsnorm_f16(
      row, spec_.hidden_size * 2, cb(final_norm), final_norm.size_bytes(),
      spec_.rms_norm_epsilon, cb(embedding), embedding.size_bytes(), cb(offsets_),
      offsets_.size_bytes(), cb(all_ids_), all_ids_.size_bytes(), mb(selected_),
      selected_.size_bytes(), nullptr, 0, mb(workspace_), workspace_.size_bytes(), 1,
      spec_.hidden_size, spec_.vocabulary_size, vs(stream)));
  if (!st.ok()) return fail<std::uint32_t>(st);
  return finish(stream);
}

}  // namespace marketforge::cuda
