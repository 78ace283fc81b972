// Per-step model inputs built on the device from the batch's persistent block tables.
//
// Reference: Worker._prepare_model_inputs (aegaeon/aegaeon/worker.py:596-682) loops over the
// batch in Python every step: for request i with context_len c and seq_len n it appends
// positions c .. n-1 and their slots table[p // 16] * 16 + p % 16 (worker.py:612-633), keeps
// the block-table row of decode requests and an empty row for prompts (worker.py:603-609),
// pads the rows with zeros (worker.py:640-646, utils.py:241-257) and builds query/sequence
// start offsets by cumulative sums (worker.py:653-676). Here:
//   * step_fused_kernel (batches of up to kFusedMaxB requests, one launch): every CTA scans the
//     batch's lengths into query start offsets in shared memory (CTA 0 also writes the offset
//     arrays, query lengths and token count), then takes its share of the new tokens: request
//     of the token by binary search in shared memory, position and slot; and its share of the
//     attention table rows (a decode row is the request's blocks, a prompt row zeros);
//   * step_scan_kernel + step_expand_kernel: the same in two launches for larger batches (one
//     CTA scans into global memory, the grid expands);
//   * table_update_kernel: applies (row, column, block id) deltas to the persistent tables, so
//     that a step uploads the blocks that changed instead of the whole padded table.
// Integer work, bit-exact with the reference's arithmetic.
#include "aeg_common.cuh"

#include <algorithm>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_step = 0;

constexpr int kBlockTokens = 16;  // tokens per KV block (Aegaeon's block size)
constexpr int kScanThreads = 1024;
constexpr int kExpandThreads = 256;

// Length of request i's new-token range, 0 (and a device error) for an invalid request.
__device__ __forceinline__ bool request_ok(int c, int n, int table_stride) {
  return c >= 0 && n >= c && static_cast<int64_t>(n) <= static_cast<int64_t>(table_stride) * kBlockTokens;
}

__device__ __forceinline__ int new_tokens(int c, int n, int table_stride) {
  if (c < 0 || n < c || static_cast<int64_t>(n) > static_cast<int64_t>(table_stride) * kBlockTokens) {
    atomicOr(&g_deverr_step, AEG_DEVERR_SEQ_LEN_RANGE);
    return 0;
  }
  return n - c;
}

__global__ void __launch_bounds__(kScanThreads)
step_scan_kernel(const int32_t* __restrict__ context_lens, const int32_t* __restrict__ seq_lens, int B,
                 int table_stride, int64_t* __restrict__ query_lens, int32_t* __restrict__ query_start_loc,
                 int32_t* __restrict__ seq_start_loc, int64_t* __restrict__ num_tokens) {
  __shared__ int64_t s_q[kScanThreads / 32], s_s[kScanThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = (B + kScanThreads - 1) / kScanThreads;
  const int i0 = min(B, tid * per), i1 = min(B, i0 + per);
  int64_t q = 0, s = 0;
  for (int i = i0; i < i1; ++i) {
    const int c = context_lens[i], n = seq_lens[i];
    const int len = new_tokens(c, n, table_stride);
    q += len;
    s += n;
  }
  // block-wide exclusive scans of (q, s)
  int64_t qi = q, si = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t tq = __shfl_up_sync(0xffffffffu, qi, o), ts = __shfl_up_sync(0xffffffffu, si, o);
    if (lane >= o) {
      qi += tq;
      si += ts;
    }
  }
  if (lane == 31) {
    s_q[wid] = qi;
    s_s[wid] = si;
  }
  __syncthreads();
  int64_t qoff = 0, soff = 0, qtot = 0, stot = 0;
  for (int w = 0; w < kScanThreads / 32; ++w) {
    if (w < wid) {
      qoff += s_q[w];
      soff += s_s[w];
    }
    qtot += s_q[w];
    stot += s_s[w];
  }
  int64_t qo = qoff + qi - q, so = soff + si - s;
  for (int i = i0; i < i1; ++i) {
    const int c = context_lens[i], n = seq_lens[i];
    const int len = (c < 0 || n < c || static_cast<int64_t>(n) > static_cast<int64_t>(table_stride) * kBlockTokens)
                        ? 0
                        : n - c;
    query_lens[i] = len;
    query_start_loc[i] = static_cast<int32_t>(qo);  // int32 as the reference's tensors (wraps alike)
    seq_start_loc[i] = static_cast<int32_t>(so);
    qo += len;
    so += n;
  }
  if (tid == 0) {
    query_start_loc[B] = static_cast<int32_t>(qtot);
    seq_start_loc[B] = static_cast<int32_t>(stot);
    *num_tokens = qtot;
  }
}

__global__ void __launch_bounds__(kExpandThreads)
step_expand_kernel(const int32_t* __restrict__ tables, int table_stride, const int32_t* __restrict__ context_lens,
                   const int32_t* __restrict__ seq_lens, const int64_t* __restrict__ query_lens, int B, const int32_t* __restrict__ query_start_loc,
                   const int64_t* __restrict__ num_tokens, int64_t* __restrict__ slot_mapping,
                   int64_t* __restrict__ positions, int64_t capacity, int32_t* __restrict__ attn_tables) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t T = *num_tokens;
  if (first == 0 && T > capacity) atomicOr(&g_deverr_step, AEG_DEVERR_SLOT_RANGE);
  const int64_t Tw = T < capacity ? T : capacity;
  for (int64_t t = first; t < Tw; t += stride) {
    // The request of token t: start[lo] <= t < start[lo + 1] at the end of the search (start[0]
    // = 0, start[B] = T > t), so request lo has new tokens even when others share its offset.
    int lo = 0, hi = B;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (static_cast<int64_t>(static_cast<uint32_t>(query_start_loc[mid])) <= t) lo = mid; else hi = mid;
    }
    const int64_t p = context_lens[lo] + (t - static_cast<int64_t>(static_cast<uint32_t>(query_start_loc[lo])));
    const int32_t blk = tables[static_cast<int64_t>(lo) * table_stride + p / kBlockTokens];
    positions[t] = p;
    slot_mapping[t] = static_cast<int64_t>(blk) * kBlockTokens + p % kBlockTokens;
  }
  if (attn_tables != nullptr) {  // a decode row keeps the blocks of its seq_len tokens, a prompt row is empty
    const int64_t cells = static_cast<int64_t>(B) * table_stride;
    for (int64_t k = first; k < cells; k += stride) {
      const int64_t i = k / table_stride, j = k - i * table_stride;
      const int64_t used = (static_cast<int64_t>(seq_lens[i]) + kBlockTokens - 1) / kBlockTokens;
      attn_tables[k] = (context_lens[i] > 0 && query_lens[i] > 0 && j < used) ? tables[k] : 0;
    }
  }
}

constexpr int kFusedThreads = 512;
constexpr int kFusedMaxB = 8192;

__global__ void __launch_bounds__(kFusedThreads)
step_fused_kernel(const int32_t* __restrict__ tables, int table_stride, const int32_t* __restrict__ context_lens,
                  const int32_t* __restrict__ seq_lens, int B, int64_t* __restrict__ slot_mapping,
                  int64_t* __restrict__ positions, int64_t capacity, int64_t* __restrict__ query_lens,
                  int32_t* __restrict__ query_start_loc, int32_t* __restrict__ seq_start_loc,
                  int32_t* __restrict__ attn_tables, int64_t* __restrict__ num_tokens) {
  __shared__ int32_t s_start[kFusedMaxB + 1];  // query start offsets (wrapped to int32 like the reference)
  __shared__ int64_t s_q[kFusedThreads / 32], s_s[kFusedThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const bool lead = blockIdx.x == 0;
  const int per = (B + kFusedThreads - 1) / kFusedThreads;
  const int i0 = min(B, tid * per), i1 = min(B, i0 + per);
  int64_t q = 0, sl = 0;
  for (int i = i0; i < i1; ++i) {
    const int c = context_lens[i], n = seq_lens[i];
    const bool ok = request_ok(c, n, table_stride);
    if (!ok && lead) atomicOr(&g_deverr_step, AEG_DEVERR_SEQ_LEN_RANGE);
    q += ok ? n - c : 0;
    sl += n;
  }
  int64_t qi = q, si = sl;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t tq = __shfl_up_sync(0xffffffffu, qi, o), ts = __shfl_up_sync(0xffffffffu, si, o);
    if (lane >= o) {
      qi += tq;
      si += ts;
    }
  }
  if (lane == 31) {
    s_q[wid] = qi;
    s_s[wid] = si;
  }
  __syncthreads();
  int64_t qo = 0, so = 0, T = 0, S = 0;
  for (int w = 0; w < kFusedThreads / 32; ++w) {
    if (w < wid) {
      qo += s_q[w];
      so += s_s[w];
    }
    T += s_q[w];
    S += s_s[w];
  }
  qo += qi - q;
  so += si - sl;
  for (int i = i0; i < i1; ++i) {
    const int c = context_lens[i], n = seq_lens[i];
    const int len = request_ok(c, n, table_stride) ? n - c : 0;
    s_start[i] = static_cast<int32_t>(qo);
    if (lead) {
      query_lens[i] = len;
      query_start_loc[i] = static_cast<int32_t>(qo);
      seq_start_loc[i] = static_cast<int32_t>(so);
    }
    qo += len;
    so += n;
  }
  if (tid == 0) {
    s_start[B] = static_cast<int32_t>(T);
    if (lead) {
      query_start_loc[B] = static_cast<int32_t>(T);
      seq_start_loc[B] = static_cast<int32_t>(S);
      *num_tokens = T;
      if (T > capacity) atomicOr(&g_deverr_step, AEG_DEVERR_SLOT_RANGE);
    }
  }
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + tid;
  const int64_t Tw = T < capacity ? T : capacity;
  for (int64_t t = first; t < Tw; t += stride) {
    // start[lo] <= t < start[lo + 1] at the end (start[0] = 0, start[B] = T > t): request lo has
    // new tokens even when others share its offset.
    int lo = 0, hi = B;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (static_cast<int64_t>(static_cast<uint32_t>(s_start[mid])) <= t) lo = mid; else hi = mid;
    }
    const int64_t p = context_lens[lo] + (t - static_cast<int64_t>(static_cast<uint32_t>(s_start[lo])));
    const int32_t blk = tables[static_cast<int64_t>(lo) * table_stride + p / kBlockTokens];
    positions[t] = p;
    slot_mapping[t] = static_cast<int64_t>(blk) * kBlockTokens + p % kBlockTokens;
  }
  if (attn_tables != nullptr) {
    const int64_t cells = static_cast<int64_t>(B) * table_stride;
    for (int64_t k = first; k < cells; k += stride) {
      const int64_t i = k / table_stride, j = k - i * table_stride;
      const int c = context_lens[i], n = seq_lens[i];
      const int64_t used = (static_cast<int64_t>(n) + kBlockTokens - 1) / kBlockTokens;
      attn_tables[k] = (c > 0 && request_ok(c, n, table_stride) && n > c && j < used) ? tables[k] : 0;
    }
  }
}

__global__ void table_update_kernel(int32_t* __restrict__ tables, int table_stride, int rows,
                                    const int32_t* __restrict__ updates, int64_t n) {
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = updates[3 * k], c = updates[3 * k + 1], v = updates[3 * k + 2];
    if (r < 0 || r >= rows || c < 0 || c >= table_stride) {
      atomicOr(&g_deverr_step, AEG_DEVERR_BLOCK_ID_RANGE);
      continue;
    }
    tables[static_cast<int64_t>(r) * table_stride + c] = v;
  }
}

}  // namespace

uint32_t deverr_read_and_clear_step(cudaStream_t s, cudaError_t* err) {
  uint32_t v = 0, zero = 0;
  *err = cudaMemcpyFromSymbolAsync(&v, g_deverr_step, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  if (*err == cudaSuccess) *err = cudaMemcpyToSymbolAsync(g_deverr_step, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  return v;
}

}  // namespace aeg

extern "C" {

int aeg_prepare_step_inputs(const int32_t* block_tables, int table_stride, const int32_t* context_lens,
                            const int32_t* seq_lens, int B, int64_t* slot_mapping, int64_t* positions,
                            int64_t capacity, int64_t* query_lens, int32_t* query_start_loc,
                            int32_t* seq_start_loc, int32_t* attn_tables, int64_t* num_tokens, void* stream) {
  AEG_CHECK_ARG(B >= 0, "prepare_step_inputs: negative batch");
  AEG_CHECK_ARG(table_stride > 0, "prepare_step_inputs: table stride must be positive");
  AEG_CHECK_ARG(capacity >= 0, "prepare_step_inputs: negative token capacity");
  AEG_CHECK_ARG(query_start_loc != nullptr && seq_start_loc != nullptr && num_tokens != nullptr,
                "prepare_step_inputs: null output pointer");
  AEG_CHECK_ARG(B == 0 || (block_tables != nullptr && context_lens != nullptr && seq_lens != nullptr &&
                           query_lens != nullptr),
                "prepare_step_inputs: null input pointer");
  AEG_CHECK_ARG(capacity == 0 || (slot_mapping != nullptr && positions != nullptr),
                "prepare_step_inputs: null slot/position output");
  AEG_CHECK_ARG(aeg::aligned(slot_mapping, 8) && aeg::aligned(positions, 8) && aeg::aligned(query_lens, 8) &&
                    aeg::aligned(num_tokens, 8),
                "prepare_step_inputs: int64 arrays must be 8-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (B <= aeg::kFusedMaxB) {
    const int64_t work = std::max<int64_t>(capacity, attn_tables != nullptr ? static_cast<int64_t>(B) * table_stride : 0);
    const int64_t want = std::max<int64_t>(1, (work + aeg::kFusedThreads - 1) / aeg::kFusedThreads);
    const int grid = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(aeg::num_sms()) * 2));
    aeg::step_fused_kernel<<<grid, aeg::kFusedThreads, 0, s>>>(block_tables, table_stride, context_lens, seq_lens, B,
                                                              slot_mapping, positions, capacity, query_lens,
                                                              query_start_loc, seq_start_loc, attn_tables, num_tokens);
    AEG_CHECK_LAUNCH("prepare_step_inputs");
    return AEG_OK;
  }
  aeg::step_scan_kernel<<<1, aeg::kScanThreads, 0, s>>>(context_lens, seq_lens, B, table_stride, query_lens,
                                                        query_start_loc, seq_start_loc, num_tokens);
  AEG_CHECK_LAUNCH("prepare_step_inputs(scan)");
  if (B == 0) return AEG_OK;
  // threads for the larger of the token bound and the attention-table cells, at most 4 CTAs per SM
  const int64_t work = std::max<int64_t>(capacity, attn_tables != nullptr ? static_cast<int64_t>(B) * table_stride : 0);
  const int64_t want = std::max<int64_t>(1, (work + aeg::kExpandThreads - 1) / aeg::kExpandThreads);
  const int grid = static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(aeg::num_sms()) * 4));
  aeg::step_expand_kernel<<<grid, aeg::kExpandThreads, 0, s>>>(block_tables, table_stride, context_lens, seq_lens,
                                                              query_lens,
                                                              B, query_start_loc, num_tokens, slot_mapping,
                                                              positions, capacity, attn_tables);
  AEG_CHECK_LAUNCH("prepare_step_inputs(expand)");
  return AEG_OK;
}

int aeg_update_block_tables(int32_t* block_tables, int table_stride, int rows, const int32_t* d_updates, int64_t n,
                            void* stream) {
  AEG_CHECK_ARG(n >= 0, "update_block_tables: negative update count");
  if (n == 0) return AEG_OK;
  AEG_CHECK_ARG(block_tables != nullptr && d_updates != nullptr, "update_block_tables: null pointer");
  AEG_CHECK_ARG(table_stride > 0 && rows >= 0, "update_block_tables: bad table shape");
  const int64_t want = (n + 255) / 256;
  const int grid = static_cast<int>(want < aeg::num_sms() * 4 ? want : aeg::num_sms() * 4);
  aeg::table_update_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(block_tables, table_stride, rows,
                                                                              d_updates, n);
  AEG_CHECK_LAUNCH("update_block_tables");
  return AEG_OK;
}

}  // extern "C"
