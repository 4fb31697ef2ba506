// Weight files into device memory (mq_read_file_to_device): the loaders' one native step.
//
// Replaces M_driver_remote_file (qwen3moe/model.mojo:156-158: n bytes at offset `off` of the weights
// file into a device buffer), which the reference's loaders call once per manifest line. Here the
// file is read with pread into two pinned staging buffers in turn while the other one's
// host-to-device copy runs on the caller's stream, so the disk (or page cache) and PCIe overlap.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

#include "common.cuh"

namespace mq {
namespace io {

constexpr size_t kChunk = 8u << 20;  // bytes per staging buffer

struct Staging {
  void *buf[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  int fd = -1;
  ~Staging() {
    for (int b = 0; b < 2; ++b) {
      if (done[b]) cudaEventDestroy(done[b]);
      if (buf[b]) cudaFreeHost(buf[b]);
    }
    if (fd >= 0) close(fd);
  }
};

}  // namespace io
}  // namespace mq

extern "C" int mq_read_file_to_device(void *dst, int64_t nbytes, const char *path, int64_t offset, void *stream) {
  MQ_REQUIRE(path, MQ_EINVAL, "mq_read_file_to_device: null path");
  MQ_REQUIRE(nbytes >= 0 && offset >= 0, MQ_EINVAL, "mq_read_file_to_device: negative size or offset");
  if (nbytes == 0) return MQ_OK;
  MQ_REQUIRE(dst, MQ_EINVAL, "mq_read_file_to_device: null destination");
  mq::io::Staging st;
  st.fd = open(path, O_RDONLY | O_CLOEXEC);
  if (st.fd < 0) return mq::fail(MQ_EIO, "mq_read_file_to_device: open %s: %s", path, strerror(errno));
  struct stat sb;
  if (fstat(st.fd, &sb) != 0) return mq::fail(MQ_EIO, "mq_read_file_to_device: stat %s: %s", path, strerror(errno));
  MQ_REQUIRE(offset + nbytes <= static_cast<int64_t>(sb.st_size), MQ_EINVAL,
             "mq_read_file_to_device: %s has %lld bytes; the range ends at %lld", path,
             static_cast<long long>(sb.st_size), static_cast<long long>(offset + nbytes));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t chunk = std::min<size_t>(mq::io::kChunk, static_cast<size_t>(nbytes));
  for (int b = 0; b < 2; ++b) {
    cudaError_t e = cudaHostAlloc(&st.buf[b], chunk, cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&st.done[b], cudaEventDisableTiming);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_read_file_to_device: staging: %s", cudaGetErrorString(e));
  }
  int64_t pos = 0;
  for (int i = 0; pos < nbytes; ++i) {
    const int b = i & 1;
    if (i >= 2) {  // the copy out of this buffer two chunks ago must be done before it is refilled
      cudaError_t e = cudaEventSynchronize(st.done[b]);
      if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_read_file_to_device: %s", cudaGetErrorString(e));
    }
    const size_t n = static_cast<size_t>(std::min<int64_t>(static_cast<int64_t>(chunk), nbytes - pos));
    size_t got = 0;
    while (got < n) {
      const ssize_t r = pread(st.fd, static_cast<uint8_t *>(st.buf[b]) + got, n - got, offset + pos + got);
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0)
        return mq::fail(MQ_EIO, "mq_read_file_to_device: read of %s at %lld: %s", path,
                        static_cast<long long>(offset + pos + got), r < 0 ? strerror(errno) : "end of file");
      got += static_cast<size_t>(r);
    }
    cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t *>(dst) + pos, st.buf[b], n, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaEventRecord(st.done[b], s);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_read_file_to_device: copy: %s", cudaGetErrorString(e));
    pos += static_cast<int64_t>(n);
  }
  // The staging buffers are freed on return: every copy out of them must have finished.
  for (int b = 0; b < 2; ++b) {
    cudaError_t e = cudaEventSynchronize(st.done[b]);
    if (e != cudaSuccess) return mq::fail(MQ_ECUDA, "mq_read_file_to_device: %s", cudaGetErrorString(e));
  }
  return MQ_OK;
}
