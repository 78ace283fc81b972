// Whole-block KV movement: copy_blocks (HBM -> HBM) and swap (HBM <-> page-locked host).
//
// Reference behaviour (aegaeon/ops/swap.cu:25-60): one cudaMemcpyAsync per block of
// `block_bytes` on the caller's stream, no checks. Here:
//   * aeg_swap       validates every id on the host, then issues one copy-engine transfer per
//                    run of blocks that are adjacent on both sides (a run of 1 is the
//                    reference's per-block copy).
//   * aeg_swap_sm    moves any number of scattered blocks with one kernel that streams 16-byte
//                    vectors between HBM and the mapped host pool (no per-block submission).
//   * aeg_copy_blocks the same kernel with both sides in HBM.
//   * aeg_migrate_blocks (migrate.cu) the same kernel between this GPU's pool and a peer GPU's
//                    pool over NVLink.
// All paths are byte copies: bit-exact for any dtype and any bit pattern.
#include "aeg_common.cuh"

#include <vector>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_copy = 0;

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 8;  // 16-byte vectors in flight per thread
constexpr int64_t kSegVecs = int64_t(kCopyThreads) * kCopyUnroll;  // 32 KiB per segment

// One work item = (pair i, segment s) of kSegVecs 16-byte vectors. Items are walked
// grid-stride so that any number of pairs needs one launch.
__global__ void __launch_bounds__(kCopyThreads)
block_copy_vec_kernel(const uint4* __restrict__ src_pool, uint4* __restrict__ dst_pool, int64_t block_vecs,
                      int64_t n_src_blocks, int64_t n_dst_blocks, const int64_t* __restrict__ src_ids,
                      const int64_t* __restrict__ dst_ids, int64_t n_pairs, int64_t segs_per_block) {
  const int64_t n_items = n_pairs * segs_per_block;
  for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int64_t pair = item / segs_per_block;
    const int64_t seg = item - pair * segs_per_block;
    const int64_t s = src_ids[pair];
    const int64_t d = dst_ids[pair];
    if (s < 0 || s >= n_src_blocks || d < 0 || d >= n_dst_blocks) {
      if (threadIdx.x == 0 && seg == 0) atomicOr(&g_deverr_copy, AEG_DEVERR_BLOCK_ID_RANGE);
      continue;
    }
    const uint4* src = src_pool + s * block_vecs;
    uint4* dst = dst_pool + d * block_vecs;
    const int64_t base = seg * kSegVecs + threadIdx.x;
    if (base + (kCopyUnroll - 1) * kCopyThreads < block_vecs) {
      uint4 v[kCopyUnroll];
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) v[u] = __ldcs(src + base + u * kCopyThreads);
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) __stcs(dst + base + u * kCopyThreads, v[u]);
    } else {
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t k = base + u * kCopyThreads;
        if (k < block_vecs) __stcs(dst + k, __ldcs(src + k));
      }
    }
  }
}

// Byte-granular variant for pools or block sizes that are not 16-byte aligned.
__global__ void __launch_bounds__(kCopyThreads)
block_copy_byte_kernel(const uint8_t* __restrict__ src_pool, uint8_t* __restrict__ dst_pool, int64_t block_bytes,
                       int64_t n_src_blocks, int64_t n_dst_blocks, const int64_t* __restrict__ src_ids,
                       const int64_t* __restrict__ dst_ids, int64_t n_pairs) {
  for (int64_t pair = blockIdx.x; pair < n_pairs; pair += gridDim.x) {
    const int64_t s = src_ids[pair];
    const int64_t d = dst_ids[pair];
    if (s < 0 || s >= n_src_blocks || d < 0 || d >= n_dst_blocks) {
      if (threadIdx.x == 0) atomicOr(&g_deverr_copy, AEG_DEVERR_BLOCK_ID_RANGE);
      continue;
    }
    const uint8_t* src = src_pool + s * block_bytes;
    uint8_t* dst = dst_pool + d * block_bytes;
    for (int64_t k = threadIdx.x; k < block_bytes; k += blockDim.x) dst[k] = src[k];
  }
}

}  // namespace

int launch_block_copy(const void* src_pool, void* dst_pool, size_t block_bytes, int64_t n_src, int64_t n_dst,
                      const int64_t* d_src, const int64_t* d_dst, int64_t n, cudaStream_t stream,
                      const char* what) {
  if (n == 0 || block_bytes == 0) return AEG_OK;
  const int sms = num_sms();
  if (block_bytes % 16 == 0 && aligned(src_pool, 16) && aligned(dst_pool, 16)) {
    const int64_t block_vecs = static_cast<int64_t>(block_bytes / 16);
    const int64_t segs = (block_vecs + kSegVecs - 1) / kSegVecs;
    const int64_t items = n * segs;
    const int64_t grid = items < int64_t(sms) * 8 ? items : int64_t(sms) * 8;
    block_copy_vec_kernel<<<static_cast<unsigned>(grid), kCopyThreads, 0, stream>>>(
        static_cast<const uint4*>(src_pool), static_cast<uint4*>(dst_pool), block_vecs, n_src, n_dst, d_src, d_dst,
        n, segs);
  } else {
    const int64_t grid = n < int64_t(sms) * 8 ? n : int64_t(sms) * 8;
    block_copy_byte_kernel<<<static_cast<unsigned>(grid), kCopyThreads, 0, stream>>>(
        static_cast<const uint8_t*>(src_pool), static_cast<uint8_t*>(dst_pool), static_cast<int64_t>(block_bytes),
        n_src, n_dst, d_src, d_dst, n);
  }
  AEG_CHECK_LAUNCH(what);
  return AEG_OK;
}

uint32_t deverr_read_and_clear_copy(cudaStream_t s, cudaError_t* err) {
  uint32_t v = 0, zero = 0;
  *err = cudaMemcpyFromSymbolAsync(&v, g_deverr_copy, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  if (*err == cudaSuccess) *err = cudaMemcpyToSymbolAsync(g_deverr_copy, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  return v;
}

}  // namespace aeg

extern "C" {

int aeg_copy_blocks(void* pool, size_t block_bytes, int64_t num_blocks, const int64_t* d_src_ids,
                    const int64_t* d_dst_ids, int64_t n, void* stream) {
  AEG_CHECK_ARG(n >= 0, "copy_blocks: negative pair count %lld", (long long)n);
  AEG_CHECK_ARG(num_blocks >= 0, "copy_blocks: negative num_blocks");
  if (n == 0) return AEG_OK;
  AEG_CHECK_ARG(pool != nullptr && d_src_ids != nullptr && d_dst_ids != nullptr, "copy_blocks: null pointer");
  AEG_CHECK_ARG(aeg::aligned(d_src_ids, 8) && aeg::aligned(d_dst_ids, 8), "copy_blocks: id arrays not 8-byte aligned");
  return aeg::launch_block_copy(pool, pool, block_bytes, num_blocks, num_blocks, d_src_ids, d_dst_ids, n,
                                static_cast<cudaStream_t>(stream), "copy_blocks");
}

int aeg_swap(void* dev_pool, void* host_pool, size_t block_bytes, int64_t n_dev_blocks, int64_t n_host_blocks,
             const int64_t* src_ids, const int64_t* dst_ids, int64_t n, int is_swap_in, void* stream) {
  AEG_CHECK_ARG(n >= 0, "swap: negative block count %lld", (long long)n);
  if (n == 0) return AEG_OK;
  AEG_CHECK_ARG(dev_pool != nullptr && host_pool != nullptr, "swap: null pool pointer");
  AEG_CHECK_ARG(src_ids != nullptr && dst_ids != nullptr, "swap: null id list");
  const int64_t n_src = is_swap_in ? n_host_blocks : n_dev_blocks;
  const int64_t n_dst = is_swap_in ? n_dev_blocks : n_host_blocks;
  for (int64_t i = 0; i < n; ++i) {
    AEG_CHECK_ARG(src_ids[i] >= 0 && src_ids[i] < n_src, "swap: source block id %lld at position %lld outside [0, %lld)",
                  (long long)src_ids[i], (long long)i, (long long)n_src);
    AEG_CHECK_ARG(dst_ids[i] >= 0 && dst_ids[i] < n_dst, "swap: target block id %lld at position %lld outside [0, %lld)",
                  (long long)dst_ids[i], (long long)i, (long long)n_dst);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* dev = static_cast<char*>(dev_pool);
  char* host = static_cast<char*>(host_pool);
  const cudaMemcpyKind kind = is_swap_in ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost;
  int64_t i = 0;
  while (i < n) {
    int64_t run = 1;
    while (i + run < n && src_ids[i + run] == src_ids[i] + run && dst_ids[i + run] == dst_ids[i] + run) ++run;
    const size_t bytes = block_bytes * static_cast<size_t>(run);
    const size_t src_off = block_bytes * static_cast<size_t>(src_ids[i]);
    const size_t dst_off = block_bytes * static_cast<size_t>(dst_ids[i]);
    if (is_swap_in) {
      AEG_CHECK_CUDA(cudaMemcpyAsync(dev + dst_off, host + src_off, bytes, kind, s));
    } else {
      AEG_CHECK_CUDA(cudaMemcpyAsync(host + dst_off, dev + src_off, bytes, kind, s));
    }
    i += run;
  }
  return AEG_OK;
}

int aeg_swap_sm(void* dev_pool, void* host_pool, size_t block_bytes, int64_t n_dev_blocks, int64_t n_host_blocks,
                const int64_t* d_src_ids, const int64_t* d_dst_ids, int64_t n, int is_swap_in, void* stream) {
  AEG_CHECK_ARG(n >= 0, "swap_sm: negative block count %lld", (long long)n);
  if (n == 0) return AEG_OK;
  AEG_CHECK_ARG(dev_pool != nullptr && host_pool != nullptr, "swap_sm: null pool pointer");
  AEG_CHECK_ARG(d_src_ids != nullptr && d_dst_ids != nullptr, "swap_sm: null id array");
  void* host_dev = nullptr;
  cudaError_t e = cudaHostGetDevicePointer(&host_dev, host_pool, 0);
  if (e != cudaSuccess || host_dev == nullptr) {
    (void)cudaGetLastError();  // clear the sticky-free error state of the failed query
    return aeg::set_error(AEG_ERR_INVALID_ARGUMENT,
                          "swap_sm: host pool %p is not page-locked and mapped (%s)", host_pool,
                          cudaGetErrorString(e));
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (is_swap_in)
    return aeg::launch_block_copy(host_dev, dev_pool, block_bytes, n_host_blocks, n_dev_blocks, d_src_ids, d_dst_ids,
                                  n, s, "swap_sm(in)");
  return aeg::launch_block_copy(dev_pool, host_dev, block_bytes, n_dev_blocks, n_host_blocks, d_src_ids, d_dst_ids, n,
                                s, "swap_sm(out)");
}

}  // extern "C"
