// GPU <-> GPU KV block migration: CUDA IPC export / open of a block pool and the whole-block
// copy between this GPU's pool and a peer GPU's pool over NVLink.
//
// Reference (stubbed there): the target engine receives the source engine's KV-cache IPC
// handles (Worker.register_kvcache_mem_handles, aegaeon/aegaeon/worker.py:860-866), opens them
// with cudaIpcOpenMemHandle and lazy peer access (aegaeon/aegaeon/cuda_wrapper.py:197-205) and
// copies each migrated request's blocks into newly allocated blocks of its own pool
// (Worker.migrate_blocks, worker.py:841-851; BlockManager._migrate_requests,
// aegaeon/aegaeon/block_manager.py:876-950). Here the copy is the block-copy kernel of
// block_copy.cu run on the current device with one pool on a peer GPU: plain 16-byte loads or
// stores over NVLink (no bulk-tensor copy ever reads peer memory), or the copy
// engines (aeg_migrate_blocks_dma).
#include "aeg_common.cuh"

#include <cuda.h>

#include <cstring>
#include <map>
#include <mutex>
#include <string>

namespace aeg {
namespace {

constexpr uint32_t kIpcMagic = 0x31474541u;  // "AEG1"

struct IpcHandle {
  cudaIpcMemHandle_t mem;  // handle of the allocation holding the pool
  int64_t offset;          // pool address - allocation base
  int64_t alloc_bytes;     // size of that allocation
  int32_t device;          // exporting device ordinal
  uint32_t magic;
  int64_t reserved;
};
static_assert(sizeof(IpcHandle) == AEG_IPC_HANDLE_BYTES, "IPC handle layout");

using GetAddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetAddressRangeFn address_range_fn() {
  static GetAddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetAddressRangeFn>(ptr);
  });
  return fn;
}

// The allocation [*base, *base + *size) that holds device address p. The driver looks it up in
// the current context: an IPC mapping lives in the importing (current) context, an allocation of
// this process on another GPU in that GPU's context, so `owner` (the device that
// cudaPointerGetAttributes names) is tried second.
int allocation_of(const void* p, int owner, uintptr_t* base, size_t* size, const char* what) {
  GetAddressRangeFn fn = address_range_fn();
  if (fn == nullptr) return set_error(AEG_ERR_CUDA, "%s: cuMemGetAddressRange is not available", what);
  CUdeviceptr b = 0;
  size_t sz = 0;
  CUresult r = fn(&b, &sz, reinterpret_cast<CUdeviceptr>(p));
  int cur = 0;
  if (r != CUDA_SUCCESS && owner >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != owner) {
    if (cudaSetDevice(owner) == cudaSuccess) {
      r = fn(&b, &sz, reinterpret_cast<CUdeviceptr>(p));
      AEG_CHECK_CUDA(cudaSetDevice(cur));
    } else {
      (void)cudaGetLastError();
    }
  }
  if (r != CUDA_SUCCESS)
    return set_error(AEG_ERR_INVALID_ARGUMENT, "%s: %p is not in a device allocation visible to this process (CUresult %d)",
                     what, p, static_cast<int>(r));
  *base = static_cast<uintptr_t>(b);
  *size = sz;
  return AEG_OK;
}

// Checks that [pool, pool + n_blocks * block_bytes) is device memory inside one allocation that
// the current device can address; enables peer access to the owning device when needed.
int check_pool(const void* pool, int64_t n_blocks, size_t block_bytes, const char* what) {
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, pool);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
    (void)cudaGetLastError();
    return set_error(AEG_ERR_INVALID_ARGUMENT, "%s: pool %p is not device memory", what, pool);
  }
  uintptr_t base = 0;
  size_t size = 0;
  int st = allocation_of(pool, attr.device, &base, &size, what);
  if (st != AEG_OK) return st;
  const uintptr_t p = reinterpret_cast<uintptr_t>(pool);
  const unsigned __int128 end = static_cast<unsigned __int128>(p) +
                                static_cast<unsigned __int128>(n_blocks) * static_cast<unsigned __int128>(block_bytes);
  if (end > static_cast<unsigned __int128>(base) + size)
    return set_error(AEG_ERR_INVALID_ARGUMENT,
                     "%s: pool %p of %lld blocks x %zu bytes runs past the end of its allocation (%zu bytes from %p)",
                     what, pool, static_cast<long long>(n_blocks), block_bytes, size, reinterpret_cast<void*>(base));
  int cur = 0;
  AEG_CHECK_CUDA(cudaGetDevice(&cur));
  if (attr.device != cur) {
    int can = 0;
    AEG_CHECK_CUDA(cudaDeviceCanAccessPeer(&can, cur, attr.device));
    if (!can)
      return set_error(AEG_ERR_UNSUPPORTED, "%s: device %d cannot address device %d's memory (no peer access)", what,
                       cur, attr.device);
    e = cudaDeviceEnablePeerAccess(attr.device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) {
      (void)cudaGetLastError();
    } else if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return set_error(AEG_ERR_CUDA, "%s: enabling peer access %d -> %d failed: %s", what, cur, attr.device,
                       cudaGetErrorString(e));
    }
  }
  return AEG_OK;
}

int check_common(const void* dst_pool, int64_t n_dst, const void* src_pool, int64_t n_src, size_t block_bytes,
                 int64_t n, const char* what) {
  AEG_CHECK_ARG(n >= 0, "%s: negative block count %lld", what, static_cast<long long>(n));
  AEG_CHECK_ARG(n_dst >= 0 && n_src >= 0, "%s: negative pool size", what);
  AEG_CHECK_ARG(dst_pool != nullptr && src_pool != nullptr, "%s: null pool pointer", what);
  AEG_CHECK_ARG(block_bytes > 0, "%s: block_bytes must be positive", what);
  return AEG_OK;
}

struct Mapping {
  void* base;
  int refs;
};
std::mutex g_ipc_mu;
std::map<std::string, Mapping> g_by_handle;      // IPC handle bytes -> mapping of the allocation
std::map<uintptr_t, std::string> g_by_pointer;   // returned pool address -> IPC handle bytes
std::map<uintptr_t, int> g_pointer_refs;         // returned pool address -> opens of that address

}  // namespace
}  // namespace aeg

extern "C" {

int aeg_ipc_export(const void* dev_pool, void* handle_out) {
  AEG_CHECK_ARG(dev_pool != nullptr && handle_out != nullptr, "ipc_export: null pointer");
  cudaPointerAttributes attr{};
  cudaError_t e = cudaPointerGetAttributes(&attr, dev_pool);
  if (e != cudaSuccess || attr.type != cudaMemoryTypeDevice) {
    (void)cudaGetLastError();
    return aeg::set_error(AEG_ERR_INVALID_ARGUMENT, "ipc_export: %p is not device memory", dev_pool);
  }
  uintptr_t base = 0;
  size_t size = 0;
  int st = aeg::allocation_of(dev_pool, attr.device, &base, &size, "ipc_export");
  if (st != AEG_OK) return st;
  aeg::IpcHandle h{};
  AEG_CHECK_CUDA(cudaIpcGetMemHandle(&h.mem, reinterpret_cast<void*>(base)));
  h.offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(dev_pool) - base);
  h.alloc_bytes = static_cast<int64_t>(size);
  h.device = attr.device;
  h.magic = aeg::kIpcMagic;
  std::memcpy(handle_out, &h, sizeof(h));
  return AEG_OK;
}

int aeg_ipc_open(const void* handle, void** dev_pool_out, int64_t* pool_bytes_out) {
  AEG_CHECK_ARG(handle != nullptr && dev_pool_out != nullptr, "ipc_open: null pointer");
  aeg::IpcHandle h;
  std::memcpy(&h, handle, sizeof(h));
  AEG_CHECK_ARG(h.magic == aeg::kIpcMagic, "ipc_open: not a handle made by aeg_ipc_export");
  AEG_CHECK_ARG(h.offset >= 0 && h.alloc_bytes > 0 && h.offset < h.alloc_bytes, "ipc_open: corrupt handle");
  const std::string key(reinterpret_cast<const char*>(&h.mem), sizeof(h.mem));
  std::lock_guard<std::mutex> lock(aeg::g_ipc_mu);
  auto it = aeg::g_by_handle.find(key);
  void* base = nullptr;
  if (it != aeg::g_by_handle.end()) {
    base = it->second.base;
    ++it->second.refs;
  } else {
    AEG_CHECK_CUDA(cudaIpcOpenMemHandle(&base, h.mem, cudaIpcMemLazyEnablePeerAccess));
    aeg::g_by_handle[key] = aeg::Mapping{base, 1};
  }
  const uintptr_t p = reinterpret_cast<uintptr_t>(base) + static_cast<uintptr_t>(h.offset);
  aeg::g_by_pointer[p] = key;
  ++aeg::g_pointer_refs[p];
  *dev_pool_out = reinterpret_cast<void*>(p);
  if (pool_bytes_out != nullptr) *pool_bytes_out = h.alloc_bytes - h.offset;
  return AEG_OK;
}

int aeg_ipc_close(void* dev_pool) {
  AEG_CHECK_ARG(dev_pool != nullptr, "ipc_close: null pointer");
  std::lock_guard<std::mutex> lock(aeg::g_ipc_mu);
  const uintptr_t p = reinterpret_cast<uintptr_t>(dev_pool);
  auto pit = aeg::g_by_pointer.find(p);
  AEG_CHECK_ARG(pit != aeg::g_by_pointer.end(), "ipc_close: %p was not returned by aeg_ipc_open", dev_pool);
  const std::string key = pit->second;
  if (--aeg::g_pointer_refs[p] == 0) {
    aeg::g_pointer_refs.erase(p);
    aeg::g_by_pointer.erase(pit);
  }
  auto it = aeg::g_by_handle.find(key);
  if (it != aeg::g_by_handle.end() && --it->second.refs == 0) {
    void* base = it->second.base;
    aeg::g_by_handle.erase(it);
    AEG_CHECK_CUDA(cudaIpcCloseMemHandle(base));
  }
  return AEG_OK;
}

int aeg_migrate_blocks(void* dst_pool, int64_t n_dst_blocks, const void* src_pool, int64_t n_src_blocks,
                       size_t block_bytes, const int64_t* d_src_ids, const int64_t* d_dst_ids, int64_t n,
                       void* stream) {
  if (n == 0) return AEG_OK;
  int st = aeg::check_common(dst_pool, n_dst_blocks, src_pool, n_src_blocks, block_bytes, n, "migrate_blocks");
  if (st != AEG_OK) return st;
  AEG_CHECK_ARG(d_src_ids != nullptr && d_dst_ids != nullptr, "migrate_blocks: null id array");
  AEG_CHECK_ARG(aeg::aligned(d_src_ids, 8) && aeg::aligned(d_dst_ids, 8), "migrate_blocks: id arrays not 8-byte aligned");
  st = aeg::check_pool(src_pool, n_src_blocks, block_bytes, "migrate_blocks(source)");
  if (st != AEG_OK) return st;
  st = aeg::check_pool(dst_pool, n_dst_blocks, block_bytes, "migrate_blocks(target)");
  if (st != AEG_OK) return st;
  return aeg::launch_block_copy(src_pool, dst_pool, block_bytes, n_src_blocks, n_dst_blocks, d_src_ids, d_dst_ids, n,
                                static_cast<cudaStream_t>(stream), "migrate_blocks");
}

int aeg_migrate_blocks_dma(void* dst_pool, int64_t n_dst_blocks, const void* src_pool, int64_t n_src_blocks,
                           size_t block_bytes, const int64_t* src_ids, const int64_t* dst_ids, int64_t n,
                           void* stream) {
  if (n == 0) return AEG_OK;
  int st = aeg::check_common(dst_pool, n_dst_blocks, src_pool, n_src_blocks, block_bytes, n, "migrate_blocks_dma");
  if (st != AEG_OK) return st;
  AEG_CHECK_ARG(src_ids != nullptr && dst_ids != nullptr, "migrate_blocks_dma: null id list");
  for (int64_t i = 0; i < n; ++i) {
    AEG_CHECK_ARG(src_ids[i] >= 0 && src_ids[i] < n_src_blocks,
                  "migrate_blocks_dma: source block id %lld at position %lld outside [0, %lld)",
                  static_cast<long long>(src_ids[i]), static_cast<long long>(i), static_cast<long long>(n_src_blocks));
    AEG_CHECK_ARG(dst_ids[i] >= 0 && dst_ids[i] < n_dst_blocks,
                  "migrate_blocks_dma: target block id %lld at position %lld outside [0, %lld)",
                  static_cast<long long>(dst_ids[i]), static_cast<long long>(i), static_cast<long long>(n_dst_blocks));
  }
  st = aeg::check_pool(src_pool, n_src_blocks, block_bytes, "migrate_blocks_dma(source)");
  if (st != AEG_OK) return st;
  st = aeg::check_pool(dst_pool, n_dst_blocks, block_bytes, "migrate_blocks_dma(target)");
  if (st != AEG_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const char* src = static_cast<const char*>(src_pool);
  char* dst = static_cast<char*>(dst_pool);
  int64_t i = 0;
  while (i < n) {
    int64_t run = 1;
    while (i + run < n && src_ids[i + run] == src_ids[i] + run && dst_ids[i + run] == dst_ids[i] + run) ++run;
    AEG_CHECK_CUDA(cudaMemcpyAsync(dst + block_bytes * static_cast<size_t>(dst_ids[i]),
                                   src + block_bytes * static_cast<size_t>(src_ids[i]),
                                   block_bytes * static_cast<size_t>(run), cudaMemcpyDefault, s));
    i += run;
  }
  return AEG_OK;
}

}  // extern "C"
