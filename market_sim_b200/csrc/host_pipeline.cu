// Native host pipeline for the ragged head: batches that live in host memory
// go H2D, through the head and back D2H, with `depth` slots in flight.  Each
// slot owns a stream, its device buffers and its own head workspace, so one
// batch is three stream-ordered operations (copy in, head, copy out) plus
// the event mf_pipeline_wait uses; a slot's next batch queues behind its
// previous one on the same stream, and batches on different slots overlap
// (copies of one with the head of another, and one head's tail with the
// next head).  All per-batch work is native, so the host keeps ahead of a
// ~20 us head.  Host buffers should be pinned: a pageable buffer makes its
// copy synchronous (still correct, no overlap).
#include <cuda_runtime.h>

#include <new>
#include <vector>

#include "mf_head.h"

namespace {

// A slot holds one batch in the packed layout of mf_pipeline_submit_packed:
// `in` = hidden fp16 [rows, H] | offsets int32 [rows + 1] | ids int32 [total]
// (ids u16 [total] for mf_pipeline_submit_packed_u16ids)
// and `out` = ids u32 [rows] | scores f32 [rows], so a packed host batch moves
// with one copy each way.
struct Slot {
  void* in = nullptr;
  void* out = nullptr;
  void* workspace = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t done = nullptr;
};

}  // namespace

struct mf_pipeline {
  int device = 0;
  const void* embedding = nullptr;
  uint64_t embedding_bytes = 0, vocab = 0, hidden_size = 0, max_rows = 0, max_ids = 0;
  std::vector<Slot> slots;
  uint64_t submitted = 0;

  uint64_t packed_bytes(uint64_t rows, uint64_t total_ids, uint64_t id_size = 4) const {
    return rows * hidden_size * 2 + (rows + 1) * 4 + total_ids * id_size;
  }
};

namespace {

mf_status st_ok() { return mf_status{MF_OK, 0}; }

// Makes the pipeline's device current for the duration of one call and
// restores the caller's device afterwards (submits launch on the slot
// streams, which belong to that device).
struct DeviceScope {
  int prev = -1;
  cudaError_t err = cudaSuccess;
  explicit DeviceScope(int dev) {
    err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
    else if (err == cudaSuccess) prev = -1;  // already current: nothing to restore
  }
  ~DeviceScope() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};
mf_status st_rt(cudaError_t e) { return mf_status{MF_CUDA_RUNTIME_FAILURE, (uint32_t)e}; }

void release(mf_pipeline* p) {
  if (!p) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  for (auto& s : p->slots) {
    if (s.stream) cudaStreamSynchronize(s.stream);
    cudaFree(s.in);
    cudaFree(s.out);
    cudaFree(s.workspace);
    if (s.done) cudaEventDestroy(s.done);
    if (s.stream) cudaStreamDestroy(s.stream);
  }
  cudaSetDevice(prev);
  delete p;
}

// The head and the copy-out of one batch already copied into slot `s`: one
// copy of ids + scores when `joined` (the caller's packed output buffer),
// else one per buffer.  Adjacent addresses alone do not make a buffer
// packed: two pinned allocations can be neighbours, and one copy across both
// is invalid.
mf_status run_and_return(mf_pipeline* p, Slot& s, uint64_t rows, uint64_t total_ids,
                         void* out_ids, void* out_scores, bool joined, uint64_t* ticket,
                         bool ids_u16 = false) {
  const uint64_t hb = rows * p->hidden_size * 2;
  char* in = static_cast<char*>(s.in);
  char* out = static_cast<char*>(s.out);
  const void* ids = total_ids ? in + hb + (rows + 1) * 4 : nullptr;
  const mf_status h =
      ids_u16 ? mf_head_restricted_csr_u16ids_f16_ex(
                    in, hb, p->embedding, p->embedding_bytes, in + hb, (rows + 1) * 4, ids,
                    total_ids * 2, out, rows * 4, out + rows * 4, rows * 4, s.workspace,
                    mf_head_workspace_bytes(rows), rows, p->hidden_size, p->vocab, 0u, s.stream)
              : mf_head_restricted_csr_f16(
                    in, hb, p->embedding, p->embedding_bytes, in + hb, (rows + 1) * 4, ids,
                    total_ids * 4, out, rows * 4, out + rows * 4, rows * 4, s.workspace,
                    mf_head_workspace_bytes(rows), rows, p->hidden_size, p->vocab, s.stream);
  if (h.code != MF_OK) return h;
  cudaError_t e =
      cudaMemcpyAsync(out_ids, out, rows * (joined ? 8 : 4), cudaMemcpyDeviceToHost, s.stream);
  if (e == cudaSuccess && out_scores && !joined)
    e = cudaMemcpyAsync(out_scores, out + rows * 4, rows * 4, cudaMemcpyDeviceToHost, s.stream);
  if (e == cudaSuccess) e = cudaEventRecord(s.done, s.stream);
  if (e != cudaSuccess) return st_rt(e);
  if (ticket) *ticket = p->submitted;
  ++p->submitted;
  return st_ok();
}

}  // namespace

extern "C" mf_status mf_pipeline_create(mf_pipeline** out, const void* embedding,
                                        uint64_t embedding_bytes, uint64_t vocab,
                                        uint64_t hidden_size, uint64_t max_rows, uint64_t max_ids,
                                        uint32_t depth) {
  if (out == nullptr || embedding == nullptr || vocab == 0 || hidden_size == 0 ||
      max_rows == 0 || depth == 0 || embedding_bytes != vocab * hidden_size * 2)
    return mf_status{MF_INVALID_ARGUMENT, 0};
  if (depth > 8 || max_rows > (uint64_t)INT32_MAX - 1 || max_ids > (uint64_t)INT32_MAX)
    return mf_status{MF_RESOURCE_LIMIT, 0};
  *out = nullptr;
  auto* p = new (std::nothrow) mf_pipeline();
  if (!p) return mf_status{MF_RESOURCE_LIMIT, 0};
  p->embedding = embedding;
  p->embedding_bytes = embedding_bytes;
  p->vocab = vocab;
  p->hidden_size = hidden_size;
  p->max_rows = max_rows;
  p->max_ids = max_ids;
  cudaError_t e = cudaGetDevice(&p->device);
  const uint64_t ws = mf_head_workspace_bytes(max_rows);
  p->slots.resize(depth);
  for (auto& s : p->slots) {
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&s.in, p->packed_bytes(max_rows, max_ids));
    if (e == cudaSuccess) e = cudaMalloc(&s.out, max_rows * 8);
    if (e == cudaSuccess) e = cudaMalloc(&s.workspace, ws);
    if (e == cudaSuccess) e = cudaMemset(s.workspace, 0, ws);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();  // the workspaces are zero before use
  if (e != cudaSuccess) {
    release(p);
    return st_rt(e);
  }
  *out = p;
  return st_ok();
}

extern "C" mf_status mf_pipeline_submit(mf_pipeline* p, const void* hidden, uint64_t rows,
                                        const void* offsets, const void* ids, uint64_t total_ids,
                                        void* out_ids, void* out_scores, uint64_t* ticket) {
  if (p == nullptr || hidden == nullptr || offsets == nullptr || out_ids == nullptr ||
      rows == 0 || (total_ids && ids == nullptr))
    return mf_status{MF_INVALID_ARGUMENT, 0};
  if (rows > p->max_rows || total_ids > p->max_ids) return mf_status{MF_RESOURCE_LIMIT, 0};
  DeviceScope scope(p->device);
  if (scope.err != cudaSuccess) return st_rt(scope.err);
  Slot& s = p->slots[p->submitted % p->slots.size()];
  const uint64_t hb = rows * p->hidden_size * 2;
  char* in = static_cast<char*>(s.in);
  cudaError_t e = cudaMemcpyAsync(in, hidden, hb, cudaMemcpyHostToDevice, s.stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(in + hb, offsets, (rows + 1) * 4, cudaMemcpyHostToDevice, s.stream);
  if (e == cudaSuccess && total_ids)
    e = cudaMemcpyAsync(in + hb + (rows + 1) * 4, ids, total_ids * 4, cudaMemcpyHostToDevice,
                        s.stream);
  if (e != cudaSuccess) return st_rt(e);
  return run_and_return(p, s, rows, total_ids, out_ids, out_scores, false, ticket);
}

extern "C" mf_status mf_pipeline_submit_packed(mf_pipeline* p, const void* batch,
                                               uint64_t batch_bytes, uint64_t rows,
                                               uint64_t total_ids, void* out,
                                               uint64_t* ticket) {
  if (p == nullptr || batch == nullptr || out == nullptr || rows == 0)
    return mf_status{MF_INVALID_ARGUMENT, 0};
  if (rows > p->max_rows || total_ids > p->max_ids) return mf_status{MF_RESOURCE_LIMIT, 0};
  if (batch_bytes != p->packed_bytes(rows, total_ids)) return mf_status{MF_INVALID_ARGUMENT, 0};
  DeviceScope scope(p->device);
  if (scope.err != cudaSuccess) return st_rt(scope.err);
  Slot& s = p->slots[p->submitted % p->slots.size()];
  const cudaError_t e =
      cudaMemcpyAsync(s.in, batch, batch_bytes, cudaMemcpyHostToDevice, s.stream);
  if (e != cudaSuccess) return st_rt(e);
  return run_and_return(p, s, rows, total_ids, out, static_cast<char*>(out) + rows * 4, true,
                        ticket);
}

extern "C" mf_status mf_pipeline_submit_packed_u16ids(mf_pipeline* p, const void* batch,
                                                      uint64_t batch_bytes, uint64_t rows,
                                                      uint64_t total_ids, void* out,
                                                      uint64_t* ticket) {
  if (p == nullptr || batch == nullptr || out == nullptr || rows == 0 || p->vocab > 65536)
    return mf_status{MF_INVALID_ARGUMENT, 0};
  if (rows > p->max_rows || total_ids > p->max_ids) return mf_status{MF_RESOURCE_LIMIT, 0};
  if (batch_bytes != p->packed_bytes(rows, total_ids, 2)) return mf_status{MF_INVALID_ARGUMENT, 0};
  DeviceScope scope(p->device);
  if (scope.err != cudaSuccess) return st_rt(scope.err);
  Slot& s = p->slots[p->submitted % p->slots.size()];
  const cudaError_t e =
      cudaMemcpyAsync(s.in, batch, batch_bytes, cudaMemcpyHostToDevice, s.stream);
  if (e != cudaSuccess) return st_rt(e);
  return run_and_return(p, s, rows, total_ids, out, static_cast<char*>(out) + rows * 4, true,
                        ticket, true);
}

extern "C" mf_status mf_pipeline_wait(mf_pipeline* p, uint64_t ticket) {
  if (p == nullptr || ticket >= p->submitted) return mf_status{MF_INVALID_ARGUMENT, 0};
  // The slot's event is re-recorded by every batch that reuses the slot, on
  // the same stream and after the ticket's own work, so waiting on it also
  // covers an older ticket whose slot has been reused since (it may wait a
  // little longer than needed, never less).
  const cudaError_t e = cudaEventSynchronize(p->slots[ticket % p->slots.size()].done);
  return e == cudaSuccess ? st_ok() : st_rt(e);
}

extern "C" mf_status mf_pipeline_synchronize(mf_pipeline* p) {
  if (p == nullptr) return mf_status{MF_INVALID_ARGUMENT, 0};
  for (auto& s : p->slots) {
    const cudaError_t e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess) return st_rt(e);
  }
  return st_ok();
}

extern "C" uint32_t mf_pipeline_depth(mf_pipeline* p) {
  return p ? (uint32_t)p->slots.size() : 0u;
}

extern "C" void* mf_pipeline_stream(mf_pipeline* p, uint32_t slot) {
  if (!p || slot >= p->slots.size()) return nullptr;
  return (void*)p->slots[slot].stream;
}

extern "C" void mf_pipeline_destroy(mf_pipeline* p) { release(p); }
