// reshape_and_cache: scatter each new token's K and V rows into its cache slot.
//
// Semantics follow vLLM 0.5.1 `reshape_and_cache_flash` as the reference reaches it per layer
// (aegaeon/aegaeon/worker.py:517-523; slots from worker.py:628-633): slot s maps to block
// s / 16, row s % 16 of the (16, Hkv, D) block interior; s < 0 is padding and is skipped.
//
// A decode step's few tokens: one CTA per token, its threads moving the token's Hkv*D key and
// value elements as 16-byte vectors (64 + 64 vectors for Hkv=4, D=128). A prompt batch's many
// tokens: one warp per token over a grid of a few CTAs per SM, each lane loading all of its
// vectors of the token before storing any, so that every resident warp keeps its token's rows in
// flight (one CTA per token leaves the GPU launching CTAs, with ~5 MB in flight). The copy is
// bit-exact either way.
#include "aeg_common.cuh"

#include <algorithm>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_cache = 0;

constexpr int kCacheThreads = 128;
constexpr int kWarpKernelThreads = 256;
constexpr int64_t kWarpKernelMinTokens = 1024;  // from this many tokens on, one warp per token

// The kernels run under programmatic dependent launch. Each first lets the next kernel launch
// and then waits for the preceding one (which may have produced the keys, values or slots)
// before reading anything: the next kernel's CTAs can then take SMs as the preceding kernel's
// leave, as they would if this launch were not between them (the decode attention after it
// requests its first tiles early and waits for this kernel before reading a row it writes; a
// kernel launched after it reads its results only after its own grid-dependency wait, which
// covers this kernel, and this kernel completes only after the one before it). Measured on the
// reference's two-call layer (cache write, then attention): a cfg2 step 1.14 x the fused one
// instead of 1.25 x, cfg3 1.02 x instead of 1.07 x. Each thread issues its first row loads
// together with the slot load, so a token costs one global round trip before its stores.
__global__ void __launch_bounds__(kCacheThreads)
reshape_and_cache_vec_kernel(const uint4* __restrict__ key, const uint4* __restrict__ value, int64_t key_stride_v,
                             int64_t value_stride_v, uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                             int64_t block_stride_v, int64_t num_slots, const int64_t* __restrict__ slot_mapping,
                             int row_vecs) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int64_t t = blockIdx.x;
  const int i0 = threadIdx.x;
  uint4 first = make_uint4(0u, 0u, 0u, 0u);
  if (i0 < row_vecs)
    first = key[t * key_stride_v + i0];
  else if (i0 < 2 * row_vecs)
    first = value[t * value_stride_v + i0 - row_vecs];
  const int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0) atomicOr(&g_deverr_cache, AEG_DEVERR_SLOT_RANGE);
    return;
  }
  const int64_t dst = (slot >> 4) * block_stride_v + (slot & 15) * row_vecs;
  if (i0 < row_vecs)
    k_cache[dst + i0] = first;
  else if (i0 < 2 * row_vecs)
    v_cache[dst + i0 - row_vecs] = first;
  for (int i = i0 + blockDim.x; i < 2 * row_vecs; i += blockDim.x) {
    if (i < row_vecs)
      k_cache[dst + i] = key[t * key_stride_v + i];
    else
      v_cache[dst + i - row_vecs] = value[t * value_stride_v + i - row_vecs];
  }
}

// Many tokens: warp w takes tokens w, w + warps, ...; its lanes load up to 4 vectors each of the
// token's K and V rows, then store them.
__global__ void __launch_bounds__(kWarpKernelThreads)
reshape_and_cache_warp_kernel(const uint4* __restrict__ key, const uint4* __restrict__ value, int64_t key_stride_v,
                              int64_t value_stride_v, uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                              int64_t block_stride_v, int64_t num_slots, const int64_t* __restrict__ slot_mapping,
                              int row_vecs, int64_t T) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kWarpKernelThreads / 32);
  for (int64_t t = (static_cast<int64_t>(blockIdx.x) * kWarpKernelThreads + threadIdx.x) >> 5; t < T; t += warps) {
    const int64_t slot = slot_mapping[t];
    if (slot >= num_slots && lane == 0) atomicOr(&g_deverr_cache, AEG_DEVERR_SLOT_RANGE);
    const bool write = slot >= 0 && slot < num_slots;
    const int64_t dst = (slot >> 4) * block_stride_v + (slot & 15) * row_vecs;
    for (int i0 = lane; i0 < 2 * row_vecs; i0 += 4 * 32) {
      uint4 r[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + 32 * u;
        if (i < row_vecs)
          r[u] = key[t * key_stride_v + i];
        else if (i < 2 * row_vecs)
          r[u] = value[t * value_stride_v + i - row_vecs];
      }
      if (write) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int i = i0 + 32 * u;
          if (i < row_vecs)
            k_cache[dst + i] = r[u];
          else if (i < 2 * row_vecs)
            v_cache[dst + i - row_vecs] = r[u];
        }
      }
    }
  }
}

// 2-byte element variant for strides or bases that are not 16-byte aligned.
__global__ void __launch_bounds__(kCacheThreads)
reshape_and_cache_elem_kernel(const uint16_t* __restrict__ key, const uint16_t* __restrict__ value,
                              int64_t key_stride, int64_t value_stride, uint16_t* __restrict__ k_cache,
                              uint16_t* __restrict__ v_cache, int64_t block_stride, int64_t num_slots,
                              const int64_t* __restrict__ slot_mapping, int row_elems) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int64_t t = blockIdx.x;
  const int64_t slot = slot_mapping[t];
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0) atomicOr(&g_deverr_cache, AEG_DEVERR_SLOT_RANGE);
    return;
  }
  const int64_t dst = (slot >> 4) * block_stride + (slot & 15) * row_elems;
  for (int i = threadIdx.x; i < row_elems; i += blockDim.x) {
    k_cache[dst + i] = key[t * key_stride + i];
    v_cache[dst + i] = value[t * value_stride + i];
  }
}

}  // namespace

uint32_t deverr_read_and_clear_cache(cudaStream_t s, cudaError_t* err) {
  uint32_t v = 0, zero = 0;
  *err = cudaMemcpyFromSymbolAsync(&v, g_deverr_cache, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  if (*err == cudaSuccess) *err = cudaMemcpyToSymbolAsync(g_deverr_cache, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  return v;
}

}  // namespace aeg

extern "C" int aeg_reshape_and_cache(const void* key, const void* value, int64_t key_stride, int64_t value_stride,
                                     void* k_cache, void* v_cache, int64_t block_stride, int64_t num_blocks,
                                     const int64_t* slot_mapping, int64_t T, int Hkv, int D, void* stream) {
  AEG_CHECK_ARG(T >= 0, "reshape_and_cache: negative token count");
  if (T == 0) return AEG_OK;
  AEG_CHECK_ARG(T <= 0x7fffffffLL, "reshape_and_cache: too many tokens (%lld)", (long long)T);
  AEG_CHECK_ARG(Hkv > 0 && D > 0, "reshape_and_cache: Hkv and D must be positive");
  AEG_CHECK_ARG(key && value && k_cache && v_cache && slot_mapping, "reshape_and_cache: null pointer");
  AEG_CHECK_ARG(num_blocks >= 0, "reshape_and_cache: negative num_blocks");
  const int64_t row = int64_t(Hkv) * D;
  AEG_CHECK_ARG(key_stride >= row && value_stride >= row, "reshape_and_cache: token stride smaller than Hkv*D");
  AEG_CHECK_ARG(block_stride >= 16 * row, "reshape_and_cache: block stride smaller than 16*Hkv*D");
  AEG_CHECK_ARG(aeg::aligned(key, 2) && aeg::aligned(value, 2) && aeg::aligned(k_cache, 2) && aeg::aligned(v_cache, 2),
                "reshape_and_cache: pointers must be 2-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t num_slots = num_blocks * 16;
  const bool vec = (row % 8 == 0) && (key_stride % 8 == 0) && (value_stride % 8 == 0) && (block_stride % 8 == 0) &&
                   aeg::aligned(key, 16) && aeg::aligned(value, 16) && aeg::aligned(k_cache, 16) &&
                   aeg::aligned(v_cache, 16);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(T));
  cfg.blockDim = dim3(aeg::kCacheThreads);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (vec && T >= aeg::kWarpKernelMinTokens) {
    int dev = 0, sms = 0;
    AEG_CHECK_CUDA(cudaGetDevice(&dev));
    AEG_CHECK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int64_t per_cta = aeg::kWarpKernelThreads / 32;
    cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((T + per_cta - 1) / per_cta, int64_t(sms) * 8)));
    cfg.blockDim = dim3(aeg::kWarpKernelThreads);
    AEG_CHECK_CUDA(cudaLaunchKernelEx(&cfg, aeg::reshape_and_cache_warp_kernel, static_cast<const uint4*>(key),
                                      static_cast<const uint4*>(value), key_stride / 8, value_stride / 8,
                                      static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), block_stride / 8,
                                      num_slots, slot_mapping, static_cast<int>(row / 8), T));
  } else if (vec) {
    AEG_CHECK_CUDA(cudaLaunchKernelEx(&cfg, aeg::reshape_and_cache_vec_kernel, static_cast<const uint4*>(key),
                                      static_cast<const uint4*>(value), key_stride / 8, value_stride / 8,
                                      static_cast<uint4*>(k_cache), static_cast<uint4*>(v_cache), block_stride / 8,
                                      num_slots, slot_mapping, static_cast<int>(row / 8)));
  } else {
    AEG_CHECK_CUDA(cudaLaunchKernelEx(&cfg, aeg::reshape_and_cache_elem_kernel, static_cast<const uint16_t*>(key),
                                      static_cast<const uint16_t*>(value), key_stride, value_stride,
                                      static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), block_stride,
                                      num_slots, slot_mapping, static_cast<int>(row)));
  }
  AEG_CHECK_LAUNCH("reshape_and_cache");
  return AEG_OK;
}
