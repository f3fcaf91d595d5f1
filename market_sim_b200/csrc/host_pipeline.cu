// Native host pipeline for the ragged head: batches that live in host memory
// go H2D on a copy stream, through the head on a compute stream, and their
// ids and scores come back D2H on a third stream, with `depth` device slots
// rotating so the copy-in of batch i + 1 overlaps the head of batch i.  All
// per-batch work is native (a handful of async CUDA calls), so the host
// keeps ahead of a ~25 us head.  Host buffers should be pinned: a pageable
// buffer makes its copy synchronous (still correct, no overlap).
#include <cuda_runtime.h>

#include <new>
#include <vector>

#include "mf_head.h"

namespace {

// A slot holds one batch in the packed layout of mf_pipeline_submit_packed:
// `in` = hidden fp16 [rows, H] | offsets int32 [rows + 1] | ids int32 [total]
// and `out` = ids u32 [rows] | scores f32 [rows], so a packed host batch moves
// with one copy each way.
struct Slot {
  void* in = nullptr;
  void* out = nullptr;
  cudaEvent_t loaded = nullptr, ran = nullptr, done = nullptr;
  bool used = false;
};

}  // namespace

struct mf_pipeline {
  int device = 0;
  const void* embedding = nullptr;
  uint64_t embedding_bytes = 0, vocab = 0, hidden_size = 0, max_rows = 0, max_ids = 0;
  cudaStream_t s_in = nullptr, s_run = nullptr, s_out = nullptr;
  void* workspace = nullptr;
  std::vector<Slot> slots;
  uint64_t submitted = 0;

  uint64_t packed_bytes(uint64_t rows, uint64_t total_ids) const {
    return rows * hidden_size * 2 + (rows + 1) * 4 + total_ids * 4;
  }
};

namespace {

mf_status st_ok() { return mf_status{MF_OK, 0}; }
mf_status st_rt(cudaError_t e) { return mf_status{MF_CUDA_RUNTIME_FAILURE, (uint32_t)e}; }

void release(mf_pipeline* p) {
  if (!p) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  for (auto& s : p->slots) {
    cudaFree(s.in);
    cudaFree(s.out);
    if (s.loaded) cudaEventDestroy(s.loaded);
    if (s.ran) cudaEventDestroy(s.ran);
    if (s.done) cudaEventDestroy(s.done);
  }
  cudaFree(p->workspace);
  if (p->s_in) cudaStreamDestroy(p->s_in);
  if (p->s_run) cudaStreamDestroy(p->s_run);
  if (p->s_out) cudaStreamDestroy(p->s_out);
  cudaSetDevice(prev);
  delete p;
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
  for (cudaStream_t* s : {&p->s_in, &p->s_run, &p->s_out})
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
  const uint64_t ws = mf_head_workspace_bytes(max_rows);
  if (e == cudaSuccess) e = cudaMalloc(&p->workspace, ws);
  if (e == cudaSuccess) e = cudaMemset(p->workspace, 0, ws);
  p->slots.resize(depth);
  for (auto& s : p->slots) {
    if (e == cudaSuccess) e = cudaMalloc(&s.in, p->packed_bytes(max_rows, max_ids));
    if (e == cudaSuccess) e = cudaMalloc(&s.out, max_rows * 8);
    for (cudaEvent_t* ev : {&s.loaded, &s.ran, &s.done})
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    release(p);
    return st_rt(e);
  }
  *out = p;
  return st_ok();
}

namespace {

// Everything after the copy-in of one batch into slot `s`: the head on the
// compute stream, then the copy-out: one copy of ids + scores when `joined`
// (the caller's packed output buffer), else one per buffer.  Adjacent
// addresses alone do not make a buffer packed: two pinned allocations can be
// neighbours, and one copy across both is invalid.
mf_status run_and_return(mf_pipeline* p, Slot& s, uint64_t rows, uint64_t total_ids,
                         void* out_ids, void* out_scores, bool joined, uint64_t* ticket) {
  cudaError_t e = cudaEventRecord(s.loaded, p->s_in);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_run, s.loaded, 0);
  if (e != cudaSuccess) return st_rt(e);
  const uint64_t hb = rows * p->hidden_size * 2;
  char* in = static_cast<char*>(s.in);
  char* out = static_cast<char*>(s.out);
  const mf_status h = mf_head_restricted_csr_f16(
      in, hb, p->embedding, p->embedding_bytes, in + hb, (rows + 1) * 4,
      total_ids ? in + hb + (rows + 1) * 4 : nullptr, total_ids * 4, out, rows * 4,
      out + rows * 4, rows * 4, p->workspace, mf_head_workspace_bytes(rows), rows,
      p->hidden_size, p->vocab, p->s_run);
  if (h.code != MF_OK) return h;
  e = cudaEventRecord(s.ran, p->s_run);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_out, s.ran, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(out_ids, out, rows * (joined ? 8 : 4), cudaMemcpyDeviceToHost, p->s_out);
  if (e == cudaSuccess && out_scores && !joined)
    e = cudaMemcpyAsync(out_scores, out + rows * 4, rows * 4, cudaMemcpyDeviceToHost, p->s_out);
  if (e == cudaSuccess) e = cudaEventRecord(s.done, p->s_out);
  if (e != cudaSuccess) return st_rt(e);
  s.used = true;
  if (ticket) *ticket = p->submitted;
  ++p->submitted;
  return st_ok();
}

}  // namespace

extern "C" mf_status mf_pipeline_submit(mf_pipeline* p, const void* hidden, uint64_t rows,
                                        const void* offsets, const void* ids, uint64_t total_ids,
                                        void* out_ids, void* out_scores, uint64_t* ticket) {
  if (p == nullptr || hidden == nullptr || offsets == nullptr || out_ids == nullptr ||
      rows == 0 || (total_ids && ids == nullptr))
    return mf_status{MF_INVALID_ARGUMENT, 0};
  if (rows > p->max_rows || total_ids > p->max_ids) return mf_status{MF_RESOURCE_LIMIT, 0};
  Slot& s = p->slots[p->submitted % p->slots.size()];
  cudaError_t e = cudaSuccess;
  if (s.used) e = cudaStreamWaitEvent(p->s_in, s.done, 0);  // slot's previous batch is home
  const uint64_t hb = rows * p->hidden_size * 2;
  char* in = static_cast<char*>(s.in);
  if (e == cudaSuccess) e = cudaMemcpyAsync(in, hidden, hb, cudaMemcpyHostToDevice, p->s_in);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(in + hb, offsets, (rows + 1) * 4, cudaMemcpyHostToDevice, p->s_in);
  if (e == cudaSuccess && total_ids)
    e = cudaMemcpyAsync(in + hb + (rows + 1) * 4, ids, total_ids * 4, cudaMemcpyHostToDevice,
                        p->s_in);
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
  Slot& s = p->slots[p->submitted % p->slots.size()];
  cudaError_t e = cudaSuccess;
  if (s.used) e = cudaStreamWaitEvent(p->s_in, s.done, 0);
  if (e == cudaSuccess) e = cudaMemcpyAsync(s.in, batch, batch_bytes, cudaMemcpyHostToDevice, p->s_in);
  if (e != cudaSuccess) return st_rt(e);
  return run_and_return(p, s, rows, total_ids, out, static_cast<char*>(out) + rows * 4, true,
                        ticket);
}

extern "C" mf_status mf_pipeline_wait(mf_pipeline* p, uint64_t ticket) {
  if (p == nullptr || ticket >= p->submitted) return mf_status{MF_INVALID_ARGUMENT, 0};
  if (p->submitted - ticket > p->slots.size()) return st_ok();  // slot reused: already home
  const cudaError_t e = cudaEventSynchronize(p->slots[ticket % p->slots.size()].done);
  return e == cudaSuccess ? st_ok() : st_rt(e);
}

extern "C" mf_status mf_pipeline_synchronize(mf_pipeline* p) {
  if (p == nullptr) return mf_status{MF_INVALID_ARGUMENT, 0};
  const cudaError_t e = cudaStreamSynchronize(p->s_out);
  return e == cudaSuccess ? st_ok() : st_rt(e);
}

extern "C" void* mf_pipeline_stream(mf_pipeline* p, uint32_t which) {
  if (!p) return nullptr;
  return which == 0 ? (void*)p->s_in : which == 1 ? (void*)p->s_run : (void*)p->s_out;
}

extern "C" void mf_pipeline_destroy(mf_pipeline* p) {
  if (p) cudaStreamSynchronize(p->s_out);
  release(p);
}
