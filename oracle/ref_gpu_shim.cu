// C-ABI shim over the reference's own CUDA restricted head — BENCHMARK
// COMPARATOR ONLY (never part of the product).
//
// Compiled by oracle/Makefile (target `refgpu`) for sm_100a together with
// the reference's unmodified sources src/cuda/greedy.cu, device_buffer.cu
// and cuda_stream.cu into oracle/_ref/libmfref_gpu.so.  bench.py's
// reference-GPU leg times marketforge::cuda::restricted_output_head_f16
// (src/cuda/greedy.cu:133-212, launched by the wrapper at :349-414) through
// the reference's own DeviceBuffer / CudaStream types on the same B200 as
// this repository's kernels.  A context owns the reference's device buffers
// (DeviceBuffer::allocate) and stream (CudaStream::create); inputs are
// copied into them device to device.
#include <cstdint>
#include <new>
#include <utility>

#include <cuda_runtime_api.h>

#include "marketforge/cuda/cuda_stream.hpp"
#include "marketforge/cuda/device_buffer.hpp"
#include "marketforge/cuda/greedy.hpp"

namespace {

using marketforge::cuda::CudaStream;
using marketforge::cuda::DeviceBuffer;

struct Ctx {
  DeviceBuffer hidden, embedding, allowed, counts, out;
  CudaStream stream;
  std::uint64_t rows = 0, hidden_size = 0, vocab = 0, max_allowed = 0;
};

bool alloc(DeviceBuffer& b, std::uint64_t bytes) {
  auto r = DeviceBuffer::allocate(bytes);
  if (!r) return false;
  b = std::move(r).value();
  return true;
}

}  // namespace

extern "C" {

void* mfrefgpu_create(std::uint64_t rows, std::uint64_t hidden_size, std::uint64_t vocab,
                      std::uint64_t max_allowed) {
  auto* c = new (std::nothrow) Ctx();
  if (c == nullptr) return nullptr;
  c->rows = rows;
  c->hidden_size = hidden_size;
  c->vocab = vocab;
  c->max_allowed = max_allowed;
  auto s = CudaStream::create();
  if (!s || !alloc(c->hidden, rows * hidden_size * 2) ||
      !alloc(c->embedding, vocab * hidden_size * 2) ||
      !alloc(c->allowed, rows * max_allowed * 4) || !alloc(c->counts, rows * 4) ||
      !alloc(c->out, rows * 4)) {
    delete c;
    return nullptr;
  }
  c->stream = std::move(s).value();
  return c;
}

// which: 0 hidden, 1 embedding, 2 allowed, 3 counts; src is device memory of
// exactly the buffer's size.
int mfrefgpu_upload(void* ctx, int which, const void* src, std::uint64_t bytes) {
  auto* c = static_cast<Ctx*>(ctx);
  DeviceBuffer* b = which == 0 ? &c->hidden : which == 1 ? &c->embedding
                  : which == 2 ? &c->allowed : which == 3 ? &c->counts : nullptr;
  if (b == nullptr || bytes != b->size_bytes()) return 1;
  const cudaError_t e = cudaMemcpy(reinterpret_cast<void*>(b->address().value), src, bytes,
                                   cudaMemcpyDeviceToDevice);
  return e == cudaSuccess ? 0 : 22;
}

// One launch of the reference's restricted_output_head_f16 on the context's
// stream; returns its ErrorCode (0 = ok).
int mfrefgpu_run(void* ctx) {
  auto* c = static_cast<Ctx*>(ctx);
  const auto st = marketforge::cuda::restricted_output_head_f16(
      c->hidden, c->embedding, c->allowed, c->counts, c->out, c->rows, c->hidden_size,
      c->vocab, c->max_allowed, c->stream.handle());
  return static_cast<int>(st.code);
}

void* mfrefgpu_stream(void* ctx) {
  return reinterpret_cast<void*>(static_cast<Ctx*>(ctx)->stream.handle().value);
}

int mfrefgpu_download(void* ctx, void* host_ids) {
  auto* c = static_cast<Ctx*>(ctx);
  const cudaError_t e = cudaMemcpy(host_ids, reinterpret_cast<void*>(c->out.address().value),
                                   c->rows * 4, cudaMemcpyDeviceToHost);
  return e == cudaSuccess ? 0 : 22;
}

void mfrefgpu_destroy(void* ctx) { delete static_cast<Ctx*>(ctx); }

}  // extern "C"
