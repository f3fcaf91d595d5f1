// CudaStream and DeviceBuffer for the marketforge::cuda interface: the
// reference's ownership and validation rules (src/cuda/cuda_stream.cu:11-49,
// src/cuda/device_buffer.cu:13-116), written over the CUDA runtime.
#include <cuda_runtime_api.h>

#include <limits>
#include <utility>

#include "marketforge/cuda/cuda_stream.hpp"
#include "marketforge/cuda/device_buffer.hpp"

namespace marketforge::cuda {
namespace {

Status runtime_status(cudaError_t e) noexcept {
  return e == cudaSuccess ? Status::success()
                          : Status::failure(ErrorCode::cuda_runtime_failure, (std::uint32_t)e);
}

cudaStream_t native(StreamHandle h) noexcept { return reinterpret_cast<cudaStream_t>(h.value); }

Status validate_copy(const void* host, std::uint64_t bytes, std::uint64_t offset,
                     std::uint64_t size, StreamHandle stream) noexcept {
  if (!stream.valid() || (bytes != 0 && host == nullptr))
    return Status::failure(ErrorCode::invalid_argument);
  if (offset > std::numeric_limits<std::uint64_t>::max() - bytes)
    return Status::failure(ErrorCode::arithmetic_overflow);
  if (offset + bytes > size) return Status::failure(ErrorCode::invalid_argument);
  return Status::success();
}

}  // namespace

Result<CudaStream> CudaStream::create() noexcept {
  cudaStream_t s = nullptr;
  const auto e = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
  if (e != cudaSuccess) return Result<CudaStream>::failure(runtime_status(e));
  return Result<CudaStream>::success(CudaStream(StreamHandle{reinterpret_cast<std::uintptr_t>(s)}));
}

CudaStream::CudaStream(CudaStream&& o) noexcept : handle_(std::exchange(o.handle_, {})) {}

CudaStream& CudaStream::operator=(CudaStream&& o) noexcept {
  if (this != &o) {
    release();
    handle_ = std::exchange(o.handle_, {});
  }
  return *this;
}

CudaStream::~CudaStream() noexcept { release(); }

Status CudaStream::synchronize() const noexcept {
  if (!handle_.valid()) return Status::failure(ErrorCode::invalid_argument);
  return runtime_status(cudaStreamSynchronize(native(handle_)));
}

void CudaStream::release() noexcept {
  if (!handle_.valid()) return;
  (void)cudaStreamDestroy(native(std::exchange(handle_, {})));
}

Result<DeviceBuffer> DeviceBuffer::allocate(std::uint64_t bytes) noexcept {
  if (bytes == 0) return Result<DeviceBuffer>::success(DeviceBuffer{});
  void* p = nullptr;
  const auto e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return Result<DeviceBuffer>::failure(runtime_status(e));
  return Result<DeviceBuffer>::success(
      DeviceBuffer(DeviceAddress{reinterpret_cast<std::uintptr_t>(p)}, bytes));
}

DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept
    : address_(std::exchange(o.address_, {})), size_bytes_(std::exchange(o.size_bytes_, 0)) {}

DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
  if (this != &o) {
    release();
    address_ = std::exchange(o.address_, {});
    size_bytes_ = std::exchange(o.size_bytes_, 0);
  }
  return *this;
}

DeviceBuffer::~DeviceBuffer() noexcept { release(); }

Status DeviceBuffer::copy_from_host_async(const void* source, std::uint64_t bytes,
                                          std::uint64_t offset, StreamHandle stream) noexcept {
  const auto v = validate_copy(source, bytes, offset, size_bytes_, stream);
  if (!v.ok() || bytes == 0) return v;
  return runtime_status(cudaMemcpyAsync(reinterpret_cast<char*>(address_.value) + offset, source,
                                        (size_t)bytes, cudaMemcpyHostToDevice, native(stream)));
}

Status DeviceBuffer::copy_to_host_async(void* destination, std::uint64_t bytes,
                                        std::uint64_t offset, StreamHandle stream) const noexcept {
  const auto v = validate_copy(destination, bytes, offset, size_bytes_, stream);
  if (!v.ok() || bytes == 0) return v;
  return runtime_status(cudaMemcpyAsync(destination,
                                        reinterpret_cast<const char*>(address_.value) + offset,
                                        (size_t)bytes, cudaMemcpyDeviceToHost, native(stream)));
}

void DeviceBuffer::release() noexcept {
  if (!address_.valid()) return;
  (void)cudaFree(reinterpret_cast<void*>(std::exchange(address_, {}).value));
  size_bytes_ = 0;
}

}  // namespace marketforge::cuda
