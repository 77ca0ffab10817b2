// Checkpoint and token-data I/O for the evaluation path.
//
//   FileStreamer          : file bytes -> device memory through two pinned chunks; the
//                           read of one chunk overlaps the DMA of the other. Used by the
//                           RSTK checkpoint loader (crates/engine/src/bin/train.rs:297-346)
//                           and the uint16 token files (crates/engine/src/data.rs:11-44),
//                           which are kept whole in HBM.
//   gather_windows_kernel : B windows of a device-resident uint16 token array ->
//                           tokens[b*S + t] = data[pos_b + t],
//                           targets[b*S + t] = data[pos_b + t + 1]
//                           (train.rs:209-211 and :556-558, `tokens(pos, seq)` and
//                           `tokens(pos + 1, seq)`).
//   eval_accumulate_kernel: per-token losses of one forward -> running sums of the loss,
//                           of the nats of byte-bearing targets and of their bytes
//                           (data.rs:75-91 compute_bpb; train.rs:197-236 validate).
#pragma once
#include <cuda_runtime.h>
#include <errno.h>
#include <stdint.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <thread>

namespace cb {

constexpr int DEV_ERR_BAD_TOKEN = 2;  // a token or target id >= vocab (same code as the embedding)

__global__ void gather_windows_kernel(const uint16_t* __restrict__ data, int64_t n,
                                      const int64_t* __restrict__ pos, int B, int S, int vocab,
                                      uint32_t* __restrict__ tokens, uint32_t* __restrict__ targets,
                                      int* err) {
  const int64_t total = (int64_t)B * S;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(i / S), t = (int)(i % S);
    const int64_t p = pos[b] + t;  // the host checked pos_b + S + 1 <= n
    uint32_t tok = p < n ? data[p] : 0u;
    uint32_t tgt = p + 1 < n ? data[p + 1] : 0u;
    if (tok >= (uint32_t)vocab || tgt >= (uint32_t)vocab) {
      atomicExch(err, DEV_ERR_BAD_TOKEN);
      tok = tok >= (uint32_t)vocab ? 0u : tok;
      tgt = tgt >= (uint32_t)vocab ? 0u : tgt;
    }
    tokens[i] = tok;
    targets[i] = tgt;
  }
}

// Running evaluation sums, updated by one block after every forward. A fixed-order
// tree over fixed per-thread strides makes the sums independent of timing.
struct EvalSums {
  double loss_sum;   // sum of all per-token losses
  double nats;       // sum of the losses of targets with a positive byte length
  long long bytes;   // sum of those byte lengths
  long long tokens;  // tokens evaluated
};

constexpr int EVAL_THREADS = 1024;

__global__ void __launch_bounds__(EVAL_THREADS)
eval_accumulate_kernel(const float* __restrict__ tok_loss, const uint32_t* __restrict__ targets,
                       const int32_t* __restrict__ token_bytes, int n_token_bytes, int T,
                       EvalSums* __restrict__ sums) {
  __shared__ double s_loss[EVAL_THREADS], s_nats[EVAL_THREADS];
  __shared__ long long s_bytes[EVAL_THREADS];
  double l = 0.0, nats = 0.0;
  long long bytes = 0;
  for (int i = threadIdx.x; i < T; i += EVAL_THREADS) {
    const float v = tok_loss[i];
    l += v;
    if (token_bytes) {
      const uint32_t tgt = targets[i];
      const int bl = tgt < (uint32_t)n_token_bytes ? token_bytes[tgt] : 0;
      if (bl > 0) {
        nats += v;
        bytes += bl;
      }
    }
  }
  s_loss[threadIdx.x] = l;
  s_nats[threadIdx.x] = nats;
  s_bytes[threadIdx.x] = bytes;
  __syncthreads();
  for (int w = EVAL_THREADS / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      s_loss[threadIdx.x] += s_loss[threadIdx.x + w];
      s_nats[threadIdx.x] += s_nats[threadIdx.x + w];
      s_bytes[threadIdx.x] += s_bytes[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    sums->loss_sum += s_loss[0];
    sums->nats += s_nats[0];
    sums->bytes += s_bytes[0];
    sums->tokens += T;
  }
}

// Streams byte ranges of an open file into device memory on one stream. Two pinned
// chunks alternate: while the DMA engine copies chunk i, the host reads chunk i+1.
// A chunk is read by READERS threads in parallel (one pread each): a single thread
// copying out of the page cache stays well below host memory bandwidth.
// Device destinations may be written asynchronously; finish() waits for all of it.
class FileStreamer {
 public:
  static constexpr size_t CHUNK = size_t(64) << 20;
  static constexpr int READERS = 8;

  FileStreamer(int fd, cudaStream_t st) : fd_(fd), st_(st) {
    for (int i = 0; i < 2; ++i) {
      if (cudaHostAlloc(&pin_[i], CHUNK, cudaHostAllocDefault) != cudaSuccess ||
          cudaEventCreateWithFlags(&ev_[i], cudaEventDisableTiming) != cudaSuccess) {
        error_ = "pinned staging allocation failed";
        return;
      }
    }
  }
  ~FileStreamer() {
    for (int i = 0; i < 2; ++i) {
      if (ev_[i]) {
        cudaEventSynchronize(ev_[i]);
        cudaEventDestroy(ev_[i]);
      }
      if (pin_[i]) cudaFreeHost(pin_[i]);
    }
  }
  bool ok() const { return error_.empty(); }
  const std::string& error() const { return error_; }
  uint64_t bytes_done() const { return done_; }

  // Enqueue the copy of file bytes [off, off + bytes) into dst (device memory).
  bool copy(void* dst, uint64_t off, uint64_t bytes) {
    char* d = static_cast<char*>(dst);
    while (ok() && bytes > 0) {
      const size_t n = bytes < CHUNK ? (size_t)bytes : CHUNK;
      const int b = next_;
      next_ ^= 1;
      if (cudaEventSynchronize(ev_[b]) != cudaSuccess) {  // the chunk's previous DMA is done
        error_ = "staging event wait failed";
        return false;
      }
      if (!read_full(pin_[b], n, off)) return false;
      if (cudaMemcpyAsync(d, pin_[b], n, cudaMemcpyHostToDevice, st_) != cudaSuccess ||
          cudaEventRecord(ev_[b], st_) != cudaSuccess) {
        error_ = "host-to-device copy failed";
        return false;
      }
      d += n;
      off += n;
      bytes -= n;
      done_ += n;
    }
    return ok();
  }

  bool finish() {
    if (ok() && cudaStreamSynchronize(st_) != cudaSuccess) error_ = "stream synchronize failed";
    return ok();
  }

 private:
  // Reads exactly n bytes at off; returns 0 or the errno of the failure (-1: end of file).
  static int pread_all(int fd, char* dst, size_t n, uint64_t off) {
    while (n > 0) {
      const ssize_t r = pread(fd, dst, n, (off_t)off);
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) return r == 0 ? -1 : errno;
      dst += r;
      off += (uint64_t)r;
      n -= (size_t)r;
    }
    return 0;
  }

  bool read_full(char* dst, size_t n, uint64_t off) {
    int err[READERS] = {0};
    const size_t part = ((n + READERS - 1) / READERS + 4095) & ~size_t(4095);
    std::thread th[READERS];
    int used = 0;
    for (size_t begin = 0; begin < n; begin += part, ++used) {
      const size_t len = std::min(part, n - begin);
      if (used == 0) continue;  // part 0 is read by this thread below
      th[used] = std::thread([=, &err] { err[used] = pread_all(fd_, dst + begin, len, off + begin); });
    }
    err[0] = pread_all(fd_, dst, std::min(part, n), off);
    for (int i = 1; i < used; ++i) th[i].join();
    for (int i = 0; i < used; ++i) {
      if (err[i] != 0) {
        error_ = err[i] < 0 ? "unexpected end of file" : std::string("read failed: ") + strerror(err[i]);
        return false;
      }
    }
    return true;
  }

  int fd_;
  cudaStream_t st_;
  char* pin_[2] = {nullptr, nullptr};
  cudaEvent_t ev_[2] = {nullptr, nullptr};
  int next_ = 0;
  uint64_t done_ = 0;
  std::string error_;
};

}  // namespace cb
