// Host side of the packed-slab loader: pread into staging and planned slice
// copies into expert parameter buffers.
//
// Same contract as spark_runtime/native/native_packed_loader.cpp (read_into
// :26-68, copy_storage_to_tensors_unlocked :70-119, the CUDA variant
// :121-174, ExpertCopyPlan::read_into_and_copy[_cuda] :232-316): argument
// checks map to DSV4_ERR_* codes (the Python layer raises the reference's
// RuntimeError messages), a failed pread keeps its errno, a short read of a
// planned block is DSV4_ERR_SHORT_READ.  Device targets get one
// cudaMemcpyAsync each on the caller's stream.
#include <cuda_runtime.h>
#include <errno.h>
#include <string.h>
#include <unistd.h>

#include <chrono>

#include "dsv4moe.h"

namespace {

int read_loop(int fd, char* dst, long long size, long long offset, long long* done, int* err_no) {
  long long completed = 0;
  while (completed < size) {
    const ssize_t r = ::pread(fd, dst + completed, static_cast<size_t>(size - completed),
                              static_cast<off_t>(offset + completed));
    if (r < 0) {
      if (errno == EINTR) continue;
      if (err_no) *err_no = errno;
      *done = completed;
      return DSV4_ERR_IO;
    }
    if (r == 0) break;
    completed += r;
  }
  *done = completed;
  return DSV4_OK;
}

int copy_slices(const char* base, long long storage_bytes, void* const* targets,
                const long long* target_bytes, const long long* offsets,
                const long long* expected, int n, int to_device, cudaStream_t st,
                long long* copied) {
  long long total = 0;
  for (int i = 0; i < n; ++i) {
    const long long off = offsets[i];
    const long long bytes = target_bytes[i];
    if (off < 0) return DSV4_ERR_ARG;
    if (expected && bytes != expected[i]) return DSV4_ERR_SIZE;
    if (off + bytes > storage_bytes) return DSV4_ERR_BOUNDS;
    if (bytes == 0) continue;
    if (to_device) {
      if (cudaMemcpyAsync(targets[i], base + off, static_cast<size_t>(bytes),
                          cudaMemcpyHostToDevice, st) != cudaSuccess)
        return DSV4_ERR_CUDA;
    } else {
      memcpy(targets[i], base + off, static_cast<size_t>(bytes));
    }
    total += bytes;
  }
  if (copied) *copied = total;
  return DSV4_OK;
}

}  // namespace

extern "C" int dsv4_read_into(int fd, void* dst, long long dst_capacity, long long size,
                              long long offset, long long* read_bytes, int* err_no) {
  if (fd < 0 || size < 0 || offset < 0 || !dst || !read_bytes) return DSV4_ERR_ARG;
  if (dst_capacity < size) return DSV4_ERR_ARG;
  return read_loop(fd, static_cast<char*>(dst), size, offset, read_bytes, err_no);
}

extern "C" int dsv4_copy_slices(const void* storage, long long storage_bytes, void* const* targets,
                                const long long* target_bytes, const long long* offsets,
                                const long long* expected_sizes, int n, int to_device,
                                void* stream, long long* copied) {
  if (!storage || n < 0 || (n > 0 && (!targets || !target_bytes || !offsets)))
    return DSV4_ERR_ARG;
  return copy_slices(static_cast<const char*>(storage), storage_bytes, targets, target_bytes,
                     offsets, expected_sizes, n, to_device, static_cast<cudaStream_t>(stream),
                     copied);
}

extern "C" int dsv4_read_into_and_copy(int fd, void* staging, long long staging_capacity,
                                       long long size, long long offset, void* const* targets,
                                       const long long* target_bytes, const long long* offsets,
                                       const long long* expected_sizes, int n, int to_device,
                                       void* stream, long long* read_bytes,
                                       long long* copied_bytes, double* read_seconds,
                                       double* copy_seconds, int* err_no) {
  if (fd < 0 || size < 0 || offset < 0 || !staging || staging_capacity < size)
    return DSV4_ERR_ARG;
  const auto t0 = std::chrono::steady_clock::now();
  long long got = 0;
  int rc = read_loop(fd, static_cast<char*>(staging), size, offset, &got, err_no);
  const auto t1 = std::chrono::steady_clock::now();
  if (read_bytes) *read_bytes = got;
  if (rc != DSV4_OK) return rc;
  if (got != size) return DSV4_ERR_SHORT_READ;
  long long copied = 0;
  rc = copy_slices(static_cast<const char*>(staging), size, targets, target_bytes, offsets,
                   expected_sizes, n, to_device, static_cast<cudaStream_t>(stream), &copied);
  const auto t2 = std::chrono::steady_clock::now();
  if (copied_bytes) *copied_bytes = copied;
  if (read_seconds) *read_seconds = std::chrono::duration<double>(t1 - t0).count();
  if (copy_seconds) *copy_seconds = std::chrono::duration<double>(t2 - t1).count();
  return rc;
}
