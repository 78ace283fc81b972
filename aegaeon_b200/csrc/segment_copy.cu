// Model-weight switch: a list of byte segments copied between two address ranges in one call
// (the page-locked host model cache -> the device weight arena).
//
// Reference: when a prefetched model is switched in, Worker copies its parameters one by one,
// `new_storage.copy_(param.untyped_storage(), non_blocking=True)` for each parameter sorted by
// address (aegaeon/aegaeon/worker.py:358-365), from the /dev/shm model cache registered with
// cudaHostRegister (aegaeon/aegaeon/loader/loader.py:187-197) into slices of the device bump
// allocator (aegaeon/aegaeon/allocator.py:54-81, 16-byte aligned). Here:
//   * copy engines: one cudaMemcpyAsync per run of segments adjacent on both sides (a packed
//     model is a few runs, not one transfer per parameter);
//   * SM engine: one kernel for all segments, grid-stride over 32 KiB chunks; a chunk finds its
//     segment by binary search over the segments' first-chunk indices (in shared memory for up
//     to kSmemSegs segments), then moves 16-byte vectors (bytes where a segment is not 16-byte
//     aligned) through the mapped host memory.
// Byte copies: bit-exact for any content.
#include "aeg_common.cuh"

#include <vector>

namespace aeg {
namespace {

constexpr int kSegThreads = 256;
constexpr int kSegUnroll = 8;
constexpr int64_t kChunkBytes = int64_t(kSegThreads) * kSegUnroll * 16;  // 32 KiB
constexpr int kSmemSegs = 4096;

struct Segment {
  int64_t src, dst, bytes, first_chunk;
};

__global__ void __launch_bounds__(kSegThreads)
segment_copy_kernel(const uint8_t* __restrict__ src_base, uint8_t* __restrict__ dst_base,
                    const Segment* __restrict__ segs, int64_t n, int64_t total_chunks) {
  __shared__ int64_t s_first[kSmemSegs + 1];
  const bool in_smem = n <= kSmemSegs;
  if (in_smem) {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s_first[i] = segs[i].first_chunk;
    if (threadIdx.x == 0) s_first[n] = total_chunks;
    __syncthreads();
  }
  for (int64_t c = blockIdx.x; c < total_chunks; c += gridDim.x) {
    int64_t lo = 0, hi = n;  // segs[lo].first_chunk <= c < first_chunk of lo + 1
    while (hi - lo > 1) {
      const int64_t mid = (lo + hi) >> 1;
      const int64_t f = in_smem ? s_first[mid] : segs[mid].first_chunk;
      if (f <= c) lo = mid; else hi = mid;
    }
    const Segment sg = segs[lo];
    const int64_t off = (c - sg.first_chunk) * kChunkBytes;
    const int64_t len = sg.bytes - off < kChunkBytes ? sg.bytes - off : kChunkBytes;
    const uint8_t* s = src_base + sg.src + off;
    uint8_t* d = dst_base + sg.dst + off;
    if (aligned(s, 16) && aligned(d, 16) && len % 16 == 0) {
      const uint4* s4 = reinterpret_cast<const uint4*>(s);
      uint4* d4 = reinterpret_cast<uint4*>(d);
      const int64_t nv = len / 16;
      uint4 v[kSegUnroll];
#pragma unroll
      for (int u = 0; u < kSegUnroll; ++u) {
        const int64_t k = threadIdx.x + u * kSegThreads;
        if (k < nv) v[u] = s4[k];
      }
#pragma unroll
      for (int u = 0; u < kSegUnroll; ++u) {
        const int64_t k = threadIdx.x + u * kSegThreads;
        if (k < nv) d4[k] = v[u];
      }
    } else {
      for (int64_t k = threadIdx.x; k < len; k += blockDim.x) d[k] = s[k];
    }
  }
}

// Device address of a buffer the current device must read or write: device memory as is,
// page-locked host memory through its mapped address.
int device_address(const void* p, const void** out, const char* what) {
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(AEG_ERR_INVALID_ARGUMENT, "copy_segments: %s %p is not known to CUDA", what, p);
  }
  if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
    *out = p;
    return AEG_OK;
  }
  if (attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr) {
    *out = attr.devicePointer;
    return AEG_OK;
  }
  return set_error(AEG_ERR_INVALID_ARGUMENT,
                   "copy_segments: %s %p is pageable host memory; the SM engine needs device or page-locked memory",
                   what, p);
}

}  // namespace
}  // namespace aeg

extern "C" {

size_t aeg_copy_segments_workspace_size(int64_t n) {
  return n <= 0 ? 0 : static_cast<size_t>(n) * sizeof(aeg::Segment);
}

int aeg_copy_segments(void* dst_base, const void* src_base, const int64_t* src_offsets, const int64_t* dst_offsets,
                      const int64_t* sizes, int64_t n, int engine, void* workspace, size_t workspace_bytes,
                      void* stream) {
  AEG_CHECK_ARG(n >= 0, "copy_segments: negative segment count");
  if (n == 0) return AEG_OK;
  AEG_CHECK_ARG(dst_base != nullptr && src_base != nullptr, "copy_segments: null base pointer");
  AEG_CHECK_ARG(src_offsets != nullptr && dst_offsets != nullptr && sizes != nullptr, "copy_segments: null segment list");
  AEG_CHECK_ARG(engine == AEG_COPY_ENGINE_DMA || engine == AEG_COPY_ENGINE_SM, "copy_segments: unknown engine %d", engine);
  for (int64_t i = 0; i < n; ++i)
    AEG_CHECK_ARG(src_offsets[i] >= 0 && dst_offsets[i] >= 0 && sizes[i] >= 0 &&
                      sizes[i] <= INT64_MAX - (src_offsets[i] > dst_offsets[i] ? src_offsets[i] : dst_offsets[i]),
                  "copy_segments: segment %lld has a negative or overflowing offset/size", static_cast<long long>(i));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const char* src = static_cast<const char*>(src_base);
  char* dst = static_cast<char*>(dst_base);
  if (engine == AEG_COPY_ENGINE_DMA) {
    int64_t i = 0;
    while (i < n) {
      int64_t bytes = sizes[i];
      int64_t j = i + 1;
      while (j < n && src_offsets[j] == src_offsets[i] + bytes && dst_offsets[j] == dst_offsets[i] + bytes) bytes += sizes[j++];
      if (bytes > 0)
        AEG_CHECK_CUDA(cudaMemcpyAsync(dst + dst_offsets[i], src + src_offsets[i], static_cast<size_t>(bytes),
                                       cudaMemcpyDefault, s));
      i = j;
    }
    return AEG_OK;
  }
  AEG_CHECK_ARG(workspace != nullptr && workspace_bytes >= aeg_copy_segments_workspace_size(n),
                "copy_segments: the SM engine needs a device workspace of %zu bytes",
                aeg_copy_segments_workspace_size(n));
  const void* src_dev = nullptr;
  const void* dst_dev = nullptr;
  int st = aeg::device_address(src_base, &src_dev, "source");
  if (st != AEG_OK) return st;
  st = aeg::device_address(dst_base, &dst_dev, "target");
  if (st != AEG_OK) return st;
  std::vector<aeg::Segment> segs(static_cast<size_t>(n));
  int64_t chunks = 0;
  for (int64_t i = 0; i < n; ++i) {
    segs[i] = aeg::Segment{src_offsets[i], dst_offsets[i], sizes[i], chunks};
    chunks += (sizes[i] + aeg::kChunkBytes - 1) / aeg::kChunkBytes;
  }
  if (chunks == 0) return AEG_OK;
  // pageable source: the call returns once the table is staged, so `segs` may go out of scope
  AEG_CHECK_CUDA(cudaMemcpyAsync(workspace, segs.data(), segs.size() * sizeof(aeg::Segment), cudaMemcpyHostToDevice, s));
  const int64_t grid = chunks < int64_t(aeg::num_sms()) * 8 ? chunks : int64_t(aeg::num_sms()) * 8;
  aeg::segment_copy_kernel<<<static_cast<unsigned>(grid), aeg::kSegThreads, 0, s>>>(
      static_cast<const uint8_t*>(src_dev), static_cast<uint8_t*>(const_cast<void*>(dst_dev)),
      static_cast<const aeg::Segment*>(workspace), n, chunks);
  AEG_CHECK_LAUNCH("copy_segments");
  return AEG_OK;
}

}  // extern "C"
