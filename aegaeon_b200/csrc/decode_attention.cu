// Paged decode attention over Aegaeon's block-table KV cache, written for sm_100a.
//
// Semantics: the decode call of the vLLM 0.5.1 FlashAttention backend that the reference runs
// per layer (flash_attn_with_kvcache(q[:, None], K_l, V_l, block_table, cache_seqlens, scale,
// causal=True) reached from aegaeon/aegaeon/worker.py:517-523, metadata from worker.py:554-713).
// One query token per sequence, so every cached key j < seq_len is visible; query head h reads
// KV head h / (Hq / Hkv).
//
// Design (memory-bound: every K/V byte is read exactly once per layer call):
//   * Work unit = (sequence b, KV head h, range of 16-token blocks). A plan kernel, run once
//     per decode step, cuts every (b, h) into ranges of near-equal length (at most kMaxSplits)
//     and orders the units longest first. A unit record also carries the sequence length and
//     the unit's first three block ids.
//   * Every warp is an independent worker (kWarps per CTA, one CTA per SM). Its first unit is
//     its warp index, later ones come from an atomic work counter (dynamic load balance; the
//     last warp to exit resets it for the next launch). It streams each (block, head) K and V
//     tile (16 tokens x 128 dims, 4 KiB each) into its own kStages-deep shared-memory ring with
//     5-D bulk-tensor TMA loads (128-byte swizzle, evict-first L2 policy) completing on
//     mbarriers. The next unit's record, block-table chunk and query rows (1-D bulk copy) are
//     prefetched one phase per processed block, and the ring keeps streaming across unit
//     boundaries. No CTA-wide barrier is taken after set-up.
//   * Per block the warp computes S^T = K Q^T with mma.sync m16n8k16 (16 tokens x 8 query
//     heads of the GQA group; K fragments by ldmatrix from the swizzled tile), an fp32 online
//     softmax in the exp2 domain with quad shuffles, transposes P in registers with movmatrix
//     and accumulates O^T += V^T P^T (V fragments by ldmatrix.trans). For bf16, P enters as a
//     bf16 value plus its bf16 rounding residue (two MMAs) so that P V keeps ~16 mantissa bits.
//   * A unit covering a whole (b, h) writes the output rows; a split unit writes an fp32
//     partial (O scaled by 2^-max, max, sum). A combine kernel, launched right after with
//     programmatic dependent launch, merges the partials of every split (b, h): one warp per
//     (b, h, query head), all of its loads in one or two round trips.
//   * Fused form (aeg_decode_layer): the warp that reads a sequence's newest block writes the
//     new token's K/V row of its head into the cache and patches it into the tile.
//   * Every mbarrier wait is bounded (2 s); a timeout raises AEG_DEVERR_WAIT_TIMEOUT and the
//     warp drains instead of hanging.
#include "aeg_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <mutex>
#include <type_traits>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_attn = 0;

constexpr int kHeadDim = 128;
constexpr int kHalves = kHeadDim / 64;  // 128-byte rows per (token, head)
constexpr int kBlockTokens = 16;
constexpr int kMaxTargetUnits = 8192;   // upper bound on the plan's balanced unit count
constexpr int kMaxSplits = 64;          // splits of one (sequence, KV head) at most
constexpr int kMinChunk = 4;            // blocks per unit at least (unless the sequence is shorter)
constexpr int kPlanThreads = 256;
constexpr int kPlanBins = 1024;         // size classes of the longest-first unit order
constexpr int kPlanCachedSeqs = 4096;   // sequences whose block counts the plan keeps in smem
constexpr uint64_t kWaitLimitNs = 2000000000ull;

constexpr int kWarps = 8;               // independent workers per CTA (one CTA per SM)
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 3;              // per-warp ring depth
constexpr int kBoxBytes = kHalves * kBlockTokens * 128;  // one (block, head) K or V tile: 4 KiB
constexpr int kStageBytes = 2 * kBoxBytes;

// Header words of the workspace.
constexpr int kHdrUnits = 0, kHdrChunk = 1, kHdrPairs = 2, kHdrSplitPairs = 3, kHdrWork = 8, kHdrExit = 9;

// ---------------------------------------------------------------------------------------
// Workspace layout (all offsets 256-byte aligned):
//   header      : int32[64]  {num_units, chunk, num_pairs, num_split_pairs, .., work, exit}
//   split_pairs : int4[P]    {pair, first unit, nsplit, 0} of every split (sequence, head)
//   units       : int4[2 * max_units]  {pair, j0, j1, (split << 16) | nsplit},
//                                      {seq_len, block id of items 0, 1, 2}
//   part_ml     : float2[max_units * G]        (max in log2 units, sum) per query head
//   part_o      : float [max_units * G * D]    partial outputs, scaled by 2^-max
struct WsLayout {
  size_t split_pairs, units, part_ml, part_o, total;
  int max_units;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

WsLayout ws_layout(int B, int Hq, int Hkv, int D) {
  WsLayout w{};
  const int G = Hq / Hkv;
  const int64_t P = int64_t(B) * Hkv;
  w.max_units = static_cast<int>(kMaxTargetUnits + P);
  size_t off = 256;
  w.split_pairs = off;
  off = align256(off + sizeof(int4) * P);
  w.units = off;
  off = align256(off + 2 * sizeof(int4) * size_t(w.max_units));
  w.part_ml = off;
  off = align256(off + sizeof(float2) * size_t(w.max_units) * G);
  w.part_o = off;
  off = align256(off + sizeof(float) * size_t(w.max_units) * G * D);
  w.total = off;
  return w;
}

struct WsPtrs {
  int* header;
  int4* split_pairs;
  int4* units;
  float2* part_ml;
  float* part_o;
};

inline WsPtrs ws_ptrs(void* ws, const WsLayout& L) {
  char* b = static_cast<char*>(ws);
  return WsPtrs{reinterpret_cast<int*>(b), reinterpret_cast<int4*>(b + L.split_pairs),
                reinterpret_cast<int4*>(b + L.units), reinterpret_cast<float2*>(b + L.part_ml),
                reinterpret_cast<float*>(b + L.part_o)};
}

// ---------------------------------------------------------------------------------------
// Plan kernel (one CTA): chunk size, split counts, unit list, split-pair list.

__device__ __forceinline__ int seq_blocks(const int* seq_lens, int b, int cap, bool report) {
  int n = seq_lens[b];
  if (n < 0 || n > cap) {
    if (report) atomicOr(&g_deverr_attn, AEG_DEVERR_SEQ_LEN_RANGE);
    n = n < 0 ? 0 : cap;
  }
  return (n + kBlockTokens - 1) / kBlockTokens;
}

__device__ __forceinline__ int splits_for(int nb, int chunk) {
  int ns = (nb + chunk - 1) / chunk;
  ns = ns < 1 ? 1 : ns;
  return ns > kMaxSplits ? kMaxSplits : ns;
}

__device__ __forceinline__ int size_bin(int nb, int chunk) {
  if (chunk < kPlanBins) return nb;
  const long long b = static_cast<long long>(nb) * (kPlanBins - 1) / chunk;
  return static_cast<int>(b);
}

// Block-wide exclusive scan of one int per thread; also returns the total.
__device__ __forceinline__ int block_excl_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) s_warp[wid] = incl;
  __syncthreads();
  int off = 0;
  total = 0;
  for (int i = 0; i < kPlanThreads / 32; ++i) {
    if (i < wid) off += s_warp[i];
    total += s_warp[i];
  }
  return off + incl - v;
}

// Unit order, longest first: all units of split (sequence, head) pairs (each about `chunk`
// blocks) in pair order, then the unsplit pairs by decreasing block count. Workers take units
// in this order, so the tail of a launch is made of the smallest ones.
__global__ void __launch_bounds__(kPlanThreads)
decode_plan_kernel(const int* __restrict__ seq_lens, const int* __restrict__ tables, int B, int Hkv,
                   int table_stride, int target_units, WsPtrs ws) {
  __shared__ long long s_red[kPlanThreads / 32];
  __shared__ int s_warp[kPlanThreads / 32];
  __shared__ int s_hist[kPlanBins];
  __shared__ int s_cursor[kPlanBins];
  __shared__ int s_nb[kPlanCachedSeqs];  // blocks per sequence (first kPlanCachedSeqs sequences)
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int P = B * Hkv;
  const int cap = table_stride * kBlockTokens;

  for (int i = tid; i < kPlanBins; i += kPlanThreads) s_hist[i] = 0;

  // Pass 1: total (block, head) items -> chunk.
  long long local = 0;
  for (int b = tid; b < B; b += kPlanThreads) {
    const int nb = seq_blocks(seq_lens, b, cap, true);
    if (b < kPlanCachedSeqs) s_nb[b] = nb;
    local += nb;
  }
  auto blocks_of = [&](int b) { return b < kPlanCachedSeqs ? s_nb[b] : seq_blocks(seq_lens, b, cap, false); };
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if (lane == 0) s_red[wid] = local;
  __syncthreads();
  long long total = 0;
  for (int i = 0; i < kPlanThreads / 32; ++i) total += s_red[i];
  total *= Hkv;
  int chunk = static_cast<int>((total + target_units - 1) / target_units);
  chunk = chunk < kMinChunk ? kMinChunk : chunk;

  // Pass 2: split units and split pairs counted over contiguous pair ranges; unsplit pairs binned.
  const int per = (P + kPlanThreads - 1) / kPlanThreads;
  const int p0 = min(P, tid * per), p1 = min(P, p0 + per);
  int cnt_units = 0, cnt_pairs = 0;
  for (int p = p0; p < p1; ++p) {
    const int nb = blocks_of(p / Hkv);
    const int ns = splits_for(nb, chunk);
    if (ns > 1) {
      cnt_units += ns;
      ++cnt_pairs;
    } else {
      atomicAdd(&s_hist[size_bin(nb, chunk)], 1);
    }
  }
  int n_split_units = 0, n_split_pairs = 0;
  int u = block_excl_scan(cnt_units, s_warp, n_split_units);
  int sp = block_excl_scan(cnt_pairs, s_warp, n_split_pairs);

  // Descending-size offsets of the bins: thread t owns bins [4t, 4t + 4); the offset of its
  // bins is the number of unsplit units in all higher bins (a reversed block scan).
  static_assert(kPlanBins == 4 * kPlanThreads, "four bins per plan thread");
  int loc[4], own = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    loc[i] = s_hist[4 * tid + i];
    own += loc[i];
  }
  __syncthreads();
  s_cursor[kPlanThreads - 1 - tid] = own;  // reversed order (scratch use of s_cursor)
  __syncthreads();
  int dummy = 0;
  const int rexcl = block_excl_scan(s_cursor[tid], s_warp, dummy);
  __syncthreads();
  s_cursor[kPlanBins - 1 - tid] = rexcl;  // units owned by threads above (kPlanThreads - 1 - tid)
  __syncthreads();
  const int higher = s_cursor[kPlanBins - 1 - (kPlanThreads - 1 - tid)];
  __syncthreads();
  int run = n_split_units + higher;
#pragma unroll
  for (int i = 3; i >= 0; --i) {
    s_cursor[4 * tid + i] = run;
    run += loc[i];
  }
  if (tid == 0) {
    ws.header[kHdrUnits] = run;  // thread 0 owns the lowest bins: its running end is the total
    ws.header[kHdrChunk] = chunk;
    ws.header[kHdrPairs] = P;
    ws.header[kHdrSplitPairs] = n_split_pairs;
    ws.header[kHdrWork] = 0;
    ws.header[kHdrExit] = 0;
  }
  __syncthreads();

  // Pass 3: write the units and the split-pair list. A unit record also carries the sequence
  // length and its first three block ids, so that a worker can request its first tiles after
  // one load.
  auto put = [&](int idx, int p, int j0, int j1, int sw) {
    const int b = p / Hkv;
    const int* tb = tables + static_cast<int64_t>(b) * table_stride + j0;
    const int n = j1 - j0;
    const int n_ctx = min(max(seq_lens[b], 0), cap);
    ws.units[2 * idx] = make_int4(p, j0, j1, sw);
    ws.units[2 * idx + 1] = make_int4(n_ctx, n > 0 ? tb[0] : 0, n > 1 ? tb[1] : 0, n > 2 ? tb[2] : 0);
  };
  for (int p = p0; p < p1; ++p) {
    const int nb = blocks_of(p / Hkv);
    const int ns = splits_for(nb, chunk);
    if (ns > 1) {
      ws.split_pairs[sp++] = make_int4(p, u, ns, 0);
      for (int s = 0; s < ns; ++s) {
        const int j0 = static_cast<int>((static_cast<long long>(s) * nb) / ns);
        const int j1 = static_cast<int>((static_cast<long long>(s + 1) * nb) / ns);
        put(u++, p, j0, j1, (s << 16) | ns);
      }
    } else {
      const int pos = atomicAdd(&s_cursor[size_bin(nb, chunk)], 1);
      put(pos, p, 0, nb, 1);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Attention kernel.

struct AttnParams {
  void* out;
  int64_t out_stride;
  const void* q;
  int64_t q_stride;
  const int* tables;
  int table_stride;
  const int* seq_lens;
  int G;
  int Hkv;
  int num_pairs;  // B * Hkv
  int max_units;  // capacity of the workspace unit list
  int64_t num_blocks;
  float scale_log2;
  int q_bulk;  // query rows are 16-byte aligned: stage them with bulk copies
  // Fused cache write (decode_layer): the new token of sequence b (position seq_len - 1) is
  // written into the cache and patched into the tile that holds it.
  int fuse_write;
  const void* k_new;
  const void* v_new;
  int64_t k_new_stride;  // token strides of k_new / v_new (elements)
  int64_t v_new_stride;
  void* k_cache;
  void* v_cache;
  int64_t block_stride;  // elements
  WsPtrs ws;
};

// A unit read from the workspace is used only if it is consistent with this call's shape; a
// workspace that was not planned for this call (or not planned at all) is skipped and reported
// instead of steering loads out of bounds.
__device__ __forceinline__ bool unit_ok(const int4& un, const int4& un1, int u, const AttnParams& p) {
  const int split = un.w >> 16, nsplit = un.w & 0xffff;
  return un.x >= 0 && un.x < p.num_pairs && un.y >= 0 && un.y <= un.z && un.z <= p.table_stride && nsplit >= 1 &&
         nsplit <= kMaxSplits && split < nsplit && u - split >= 0 && u - split + nsplit <= p.max_units &&
         un1.x >= 0 && un1.x <= p.table_stride * kBlockTokens && un.z * kBlockTokens < un1.x + kBlockTokens;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int NT>
struct AttnSmem {
  static constexpr int kQSlot = 8 * NT * kHeadDim * 2;           // query rows of one unit
  static constexpr int kPerWarp = kStages * kStageBytes + kQSlot;  // multiple of 1024
  static constexpr int kOffBars = kWarps * kPerWarp;
  static constexpr int kBarsPerWarp = kStages + 1;
  static constexpr int kTotal = kOffBars + kWarps * kBarsPerWarp * 8;
  static constexpr size_t kDynamic = size_t(kTotal) + 1024;  // + alignment slack
  static_assert(kPerWarp % 1024 == 0, "per-warp regions must keep 1024-byte alignment");
};

// One work unit as a warp sees it (all lanes hold the same values, except `tbl`, `knew`, `vnew`).
struct Unit {
  int u;        // unit index, -1 = none (queue exhausted)
  int b, h, j0, n, split, nsplit, n_ctx;
  int tbl;      // this lane's block id of the table chunk starting at item `tbase`
  int tbase;
  int issued;   // items whose tiles were requested
  int bf0, bf1, bf2;  // block ids of items 0..2 (from the unit record)
  int blk_last; // block id of the last item (fused cache write)
  int last;     // the unit holds the sequence's newest token (fused cache write)
  uint2 knew;   // this lane's 4 elements of the new K / V row of head h (fused cache write)
  uint2 vnew;
};

__device__ __forceinline__ void unit_clear(Unit& x) {
  x.u = -1;
  x.b = x.h = x.j0 = x.n = x.split = x.n_ctx = 0;
  x.nsplit = 1;
  x.tbl = x.tbase = x.issued = 0;
  x.bf0 = x.bf1 = x.bf2 = x.blk_last = 0;
  x.last = 0;
  x.knew = x.vnew = make_uint2(0u, 0u);
}

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 1)
decode_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const AttnParams p) {
  using SL = AttnSmem<NT>;
  constexpr bool kSplitP = std::is_same<T, __nv_bfloat16>::value;
  using Mma = MmaF32<T>;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  uint8_t* ring = smem + warp * SL::kPerWarp;
  T* qslot = reinterpret_cast<T*>(ring + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + SL::kOffBars) + warp * SL::kBarsPerWarp;
  uint64_t* qbar = full + kStages;

  if (lane == 0) {
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    mbar_init(qbar, 1);
    fence_mbar_init();
    if (warp == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
  }
  __syncwarp();

  // Everything below reads data produced by earlier work on the stream.
  pdl_wait_primary();
  pdl_launch_dependents();

  const int num_units = min(max(p.ws.header[kHdrUnits], 0), p.max_units);
  const int G = p.G;
  const int Hkv = p.Hkv;
  const uint64_t pol = l2_policy_evict_first();
  const T* q = static_cast<const T*>(p.q);
  T* out = static_cast<T*>(p.out);
  const int lr = lane & 7;    // row within an 8x8 matrix
  const int lm = lane >> 3;   // which of the four matrices this lane addresses
  const int quad = lane & 3;  // column pair of the accumulator fragment
  const int grp = lane >> 2;  // row of the accumulator fragment

  bool abort = false;
  uint32_t g_iss = 0, g_con = 0;  // tiles requested / consumed by this warp
  uint32_t q_phase = 0;

  auto report_timeout = [&]() {
    abort = true;
    if (lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_WAIT_TIMEOUT);
  };

  // Unit fetch in three phases so that its latency overlaps the processing of blocks:
  // A) reserve a unit index, B) load its record, C) unpack it, load the table chunk (and the
  // new K/V row for the fused write) and start the bulk copy of its query rows.
  // The first unit of every warp is its global warp index; later ones come from the counter.
  const int total_warps = static_cast<int>(gridDim.x) * kWarps;
  bool first_fetch = true;
  auto phase_a = [&]() -> int {
    int u = 0;
    if (first_fetch) {
      u = static_cast<int>(blockIdx.x) * kWarps + warp;
      first_fetch = false;
    } else if (lane == 0) {
      u = total_warps + atomicAdd(&p.ws.header[kHdrWork], 1);
    }
    return u;
  };
  auto phase_b = [&](int u_raw, int4& un1) -> int4 {
    const int u = __shfl_sync(0xffffffffu, u_raw, 0);
    if (u >= num_units) {
      un1 = make_int4(0, 0, 0, 0);
      return make_int4(-1, u, 0, 0);
    }
    un1 = p.ws.units[2 * u + 1];
    return p.ws.units[2 * u];
  };
  auto phase_c = [&](int u_raw, const int4& un, const int4& un1, Unit& x) -> bool {  // false: invalid, refetch
    const int u = __shfl_sync(0xffffffffu, u_raw, 0);
    unit_clear(x);
    if (u >= num_units) return true;  // x.u = -1: nothing left
    if (!unit_ok(un, un1, u, p)) {
      if (lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_PLAN_MISMATCH);
      return false;
    }
    x.u = u;
    x.b = un.x / Hkv;
    x.h = un.x % Hkv;
    x.j0 = un.y;
    x.n = un.z - un.y;
    x.split = un.w >> 16;
    x.nsplit = un.w & 0xffff;
    x.n_ctx = un1.x;
    x.bf0 = un1.y;
    x.bf1 = un1.z;
    x.bf2 = un1.w;
    // table chunk for items 3 .. 34 (items 0..2 come with the record)
    const int* tb = p.tables + static_cast<int64_t>(x.b) * p.table_stride + x.j0 + 3;
    x.tbase = 3;
    x.tbl = lane < min(32, x.n - 3) ? tb[lane] : 0;
    if (p.fuse_write && x.n > 0 && x.n_ctx > 0 && x.j0 + x.n == (x.n_ctx + kBlockTokens - 1) / kBlockTokens) {
      // This unit reads the block of position n_ctx - 1: keep the new K/V row of head h to
      // store it in the cache and patch it into the tile when that block is processed.
      x.last = 1;
      const uint32_t* kn = reinterpret_cast<const uint32_t*>(static_cast<const T*>(p.k_new) +
                                                             static_cast<int64_t>(x.b) * p.k_new_stride +
                                                             static_cast<int64_t>(x.h) * kHeadDim) + 2 * lane;
      const uint32_t* vn = reinterpret_cast<const uint32_t*>(static_cast<const T*>(p.v_new) +
                                                             static_cast<int64_t>(x.b) * p.v_new_stride +
                                                             static_cast<int64_t>(x.h) * kHeadDim) + 2 * lane;
      x.knew = make_uint2(kn[0], kn[1]);
      x.vnew = make_uint2(vn[0], vn[1]);
    }
    // query rows of this unit into the (now free) query slot
    const T* qsrc = q + static_cast<int64_t>(x.b) * p.q_stride + static_cast<int64_t>(x.h) * G * kHeadDim;
    const uint32_t qbytes = G * kHeadDim * 2;
    fence_proxy_async_smem();
    if (p.q_bulk) {
      if (lane == 0) {
        mbar_arrive_expect_tx(qbar, qbytes);
        bulk_load_1d(qslot, qsrc, qbytes, qbar);
      }
    } else {
      for (int i = lane; i < G * kHeadDim / 2; i += 32)
        reinterpret_cast<uint32_t*>(qslot)[i] = reinterpret_cast<const uint32_t*>(qsrc)[i];
      __syncwarp();
      if (lane == 0) mbar_arrive(qbar);
    }
    return true;
  };
  auto fetch_now = [&](Unit& x) {
    while (true) {
      const int ur = phase_a();
      int4 un1;
      const int4 un = phase_b(ur, un1);
      if (phase_c(ur, un, un1, x)) return;
    }
  };

  // Requests the next tile of unit x into the ring.
  auto issue = [&](Unit& x) {
    const int k = x.issued;
    int blk;
    if (k < 3) {
      blk = k == 0 ? x.bf0 : (k == 1 ? x.bf1 : x.bf2);
    } else {
      if (k - x.tbase >= 32) {
        x.tbase = k;
        const int* tb = p.tables + static_cast<int64_t>(x.b) * p.table_stride + x.j0 + k;
        x.tbl = lane < min(32, x.n - k) ? tb[lane] : 0;
      }
      blk = __shfl_sync(0xffffffffu, x.tbl, k - x.tbase);
    }
    if (k == x.n - 1) x.blk_last = blk;
    fence_proxy_async_smem();  // the stage being refilled was read through the generic proxy
    if (lane == 0) {
      if (static_cast<unsigned long long>(static_cast<long long>(blk)) >= static_cast<unsigned long long>(p.num_blocks))
        atomicOr(&g_deverr_attn, AEG_DEVERR_BLOCK_ID_RANGE);  // TMA zero-fills it
      if (!abort) {
        const uint32_t st = g_iss % kStages;
        uint8_t* dst = ring + st * kStageBytes;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        tma_load_5d(dst, &kmap, &full[st], 0, 0, 0, x.h, blk, pol);
        tma_load_5d(dst + kBoxBytes, &vmap, &full[st], 0, 0, 0, x.h, blk, pol);
      }
    }
    ++g_iss;
    ++x.issued;
  };

  Unit cur, nxt;
  unit_clear(nxt);
  fetch_now(cur);
  while (cur.u >= 0 && cur.issued < cur.n && g_iss - g_con < kStages) issue(cur);

  while (cur.u >= 0) {
    // Query fragments (B operand of S^T = K Q^T) from the query slot.
    if (!abort && !mbar_wait_bounded(qbar, q_phase, kWaitLimitNs)) report_timeout();
    q_phase ^= 1;
    uint32_t qf[NT][8][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int head = nt * 8 + grp;
      const bool hv = head < G;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int d = ks * 16 + 2 * quad;
        qf[nt][ks][0] = hv ? *reinterpret_cast<const uint32_t*>(qslot + head * kHeadDim + d) : 0u;
        qf[nt][ks][1] = hv ? *reinterpret_cast<const uint32_t*>(qslot + head * kHeadDim + d + 8) : 0u;
      }
    }
    __syncwarp();

    float o[8][NT][4];
    float m[NT][2], l[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
    }

    // Prefetch state of the next unit.
    int pf = 0, nxt_raw = 0;
    int4 nxt_un = make_int4(0, 0, 0, 0), nxt_un1 = make_int4(0, 0, 0, 0);
    bool nxt_ready = false;
    auto prefetch_step = [&]() {
      if (pf == 0) {
        nxt_raw = phase_a();
      } else if (pf == 1) {
        nxt_un = phase_b(nxt_raw, nxt_un1);
      } else if (pf == 2) {
        if (phase_c(nxt_raw, nxt_un, nxt_un1, nxt)) {
          nxt_ready = true;
        } else {
          pf = -1;  // invalid unit: start over (reported already)
        }
      }
      if (pf < 3) ++pf;
    };
    auto refill = [&]() {
      while (g_iss - g_con < kStages) {
        if (cur.issued < cur.n)
          issue(cur);
        else if (nxt_ready && nxt.u >= 0 && nxt.issued < nxt.n)
          issue(nxt);
        else
          break;
      }
    };

    for (int k = 0; k < cur.n; ++k) {
      const uint32_t st = g_con % kStages, ph = (g_con / kStages) & 1;
      if (!abort && !mbar_wait_bounded(&full[st], ph, kWaitLimitNs)) report_timeout();
      const int j = cur.j0 + k;
      const int nvalid = min(kBlockTokens, cur.n_ctx - j * kBlockTokens);
      if (!abort && nvalid > 0) {
        const uint32_t kbase = smem_u32(ring + st * kStageBytes);
        const uint32_t vbase = kbase + kBoxBytes;
        if (cur.last && k == cur.n - 1) {
          // Fused cache write: store the newest token's K/V row of head h in the cache (no other
          // reader of that row in this launch: other warps read other heads' rows) and patch it
          // into the swizzled tiles, which were fetched before the store.
          const int t = (cur.n_ctx - 1) % kBlockTokens;
          if (static_cast<unsigned long long>(static_cast<long long>(cur.blk_last)) <
              static_cast<unsigned long long>(p.num_blocks)) {
            const int64_t off = static_cast<int64_t>(cur.blk_last) * p.block_stride +
                                (static_cast<int64_t>(t) * Hkv + cur.h) * kHeadDim + 4 * lane;
            *reinterpret_cast<uint2*>(static_cast<T*>(p.k_cache) + off) = cur.knew;
            *reinterpret_cast<uint2*>(static_cast<T*>(p.v_cache) + off) = cur.vnew;
          }
          const int half = lane >> 4, ch = (lane & 15) >> 1;
          const uint32_t soff = (half * kBlockTokens + t) * 128 + ((ch ^ (t & 7)) << 4) + (lane & 1) * 8;
          *reinterpret_cast<uint2*>(ring + st * kStageBytes + soff) = cur.knew;
          *reinterpret_cast<uint2*>(ring + st * kStageBytes + kBoxBytes + soff) = cur.vnew;
          __syncwarp();
        }

        // S^T[16 tokens][8 heads] per n-tile.
        float s[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int tok = lr + ((lm & 1) << 3);
          const int c = ks * 2 + (lm >> 1);
          const uint32_t addr = kbase + ((c >> 3) * kBlockTokens + tok) * 128 + (((c & 7) ^ lr) << 4);
          uint32_t a[4];
          ldmatrix_x4(a, addr);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) Mma::run(s[nt], a, qf[nt][ks][0], qf[nt][ks][1]);
        }

        // Online softmax (log2 domain). Column = query head, rows = tokens.
        uint32_t pb[NT][2];
        uint32_t pl[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const bool v0 = grp < nvalid, v1 = grp + 8 < nvalid;
          const float x0 = v0 ? s[nt][0] * p.scale_log2 : -INFINITY;
          const float x1 = v0 ? s[nt][1] * p.scale_log2 : -INFINITY;
          const float x2 = v1 ? s[nt][2] * p.scale_log2 : -INFINITY;
          const float x3 = v1 ? s[nt][3] * p.scale_log2 : -INFINITY;
          float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
          }
          const float mn0 = fmaxf(m[nt][0], mx0), mn1 = fmaxf(m[nt][1], mx1);
          const float a0 = ex2(m[nt][0] - mn0), a1 = ex2(m[nt][1] - mn1);
          const float p0 = ex2(x0 - mn0), p1 = ex2(x1 - mn1);
          const float p2 = ex2(x2 - mn0), p3 = ex2(x3 - mn1);
          m[nt][0] = mn0;
          m[nt][1] = mn1;
          l[nt][0] = l[nt][0] * a0 + (p0 + p2);
          l[nt][1] = l[nt][1] * a1 + (p1 + p3);
#pragma unroll
          for (int mt = 0; mt < 8; ++mt) {
            o[mt][nt][0] *= a0;
            o[mt][nt][1] *= a1;
            o[mt][nt][2] *= a0;
            o[mt][nt][3] *= a1;
          }
          const uint32_t h01 = pack2<T>(p0, p1), h23 = pack2<T>(p2, p3);
          pb[nt][0] = movmatrix_trans(h01);
          pb[nt][1] = movmatrix_trans(h23);
          if constexpr (kSplitP) {
            const float2 r01 = unpack2<T>(h01), r23 = unpack2<T>(h23);
            pl[nt][0] = movmatrix_trans(pack2<T>(p0 - r01.x, p1 - r01.y));
            pl[nt][1] = movmatrix_trans(pack2<T>(p2 - r23.x, p3 - r23.y));
          }
        }

        // O^T[128 dims][8 heads] += V^T P^T.
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int tok = lr + ((lm >> 1) << 3);
          const int c = mt * 2 + (lm & 1);
          const uint32_t addr = vbase + ((c >> 3) * kBlockTokens + tok) * 128 + (((c & 7) ^ lr) << 4);
          uint32_t a[4];
          ldmatrix_x4_trans(a, addr);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            Mma::run(o[mt][nt], a, pb[nt][0], pb[nt][1]);
            if constexpr (kSplitP) Mma::run(o[mt][nt], a, pl[nt][0], pl[nt][1]);
          }
        }
      }
      __syncwarp();
      ++g_con;
      prefetch_step();
      refill();
    }
    while (pf < 3) prefetch_step();
    refill();

    // ---- unit result ----
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        l[nt][0] += __shfl_xor_sync(0xffffffffu, l[nt][0], off);
        l[nt][1] += __shfl_xor_sync(0xffffffffu, l[nt][1], off);
      }
    if (cur.nsplit == 1) {
      T* ob = out + static_cast<int64_t>(cur.b) * p.out_stride + static_cast<int64_t>(cur.h) * G * kHeadDim;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h0 = nt * 8 + 2 * quad;
        const float i0 = l[nt][0] > 0.f ? 1.f / l[nt][0] : 0.f;
        const float i1 = l[nt][1] > 0.f ? 1.f / l[nt][1] : 0.f;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + grp;
          if (h0 < G) {
            ob[h0 * kHeadDim + d0] = from_float<T>(o[mt][nt][0] * i0);
            ob[h0 * kHeadDim + d0 + 8] = from_float<T>(o[mt][nt][2] * i0);
          }
          if (h0 + 1 < G) {
            ob[(h0 + 1) * kHeadDim + d0] = from_float<T>(o[mt][nt][1] * i1);
            ob[(h0 + 1) * kHeadDim + d0 + 8] = from_float<T>(o[mt][nt][3] * i1);
          }
        }
      }
    } else {
      const int64_t base = static_cast<int64_t>(cur.u) * G;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h0 = nt * 8 + 2 * quad;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + grp;
          if (h0 < G) {
            float* po = p.ws.part_o + (base + h0) * kHeadDim;
            po[d0] = o[mt][nt][0];
            po[d0 + 8] = o[mt][nt][2];
          }
          if (h0 + 1 < G) {
            float* po = p.ws.part_o + (base + h0 + 1) * kHeadDim;
            po[d0] = o[mt][nt][1];
            po[d0 + 8] = o[mt][nt][3];
          }
        }
        if (grp == 0) {
          if (h0 < G) p.ws.part_ml[base + h0] = make_float2(m[nt][0], l[nt][0]);
          if (h0 + 1 < G) p.ws.part_ml[base + h0 + 1] = make_float2(m[nt][1], l[nt][1]);
        }
      }
    }

    cur = nxt;
    unit_clear(nxt);
    refill();
  }

  // The last warp of the grid to finish resets the work counters for the next launch.
  if (lane == 0) {
    __threadfence();
    const int done = atomicAdd(&p.ws.header[kHdrExit], 1);
    if (done == total_warps - 1) {
      p.ws.header[kHdrWork] = 0;
      p.ws.header[kHdrExit] = 0;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Combine kernel: merges the partials of every split (sequence, KV head). Work item =
// (split pair, query head n of its group), one warp each, no block-level synchronisation:
// lane c owns float4 column c of the 128-dim row and loads that column of kCombineBatch splits
// at a time in the same round trip as the splits' (max, sum) pairs; the weights 2^(m_s - M) / L
// are exchanged by shuffles.

constexpr int kCombineThreads = 128;
constexpr int kCombineWarps = kCombineThreads / 32;
constexpr int kCombineBatch = 32;

template <typename T>
__global__ void __launch_bounds__(kCombineThreads)
decode_combine_kernel(void* out_v, int64_t out_stride, int G, int Hkv, WsPtrs ws) {
  T* out = static_cast<T*>(out_v);
  const int lane = threadIdx.x & 31;
  const int gw = static_cast<int>(blockIdx.x) * kCombineWarps + (threadIdx.x >> 5);
  const int n_warps = static_cast<int>(gridDim.x) * kCombineWarps;
  // The split-pair list comes from the plan kernel, which finished before the attention launch
  // this kernel depends on started; it is read before waiting for the attention results.
  const int n_items = ws.header[kHdrSplitPairs] * G;
  int4 sp = gw < n_items ? ws.split_pairs[gw / G] : make_int4(0, 0, 0, 0);
  pdl_wait_primary();
  pdl_launch_dependents();
  const float4* po4 = reinterpret_cast<const float4*>(ws.part_o);
  for (int item = gw; item < n_items; item += n_warps) {
    const int n = item % G;
    const int ns = min(sp.z, kMaxSplits);
    const int64_t row0 = static_cast<int64_t>(sp.y) * G + n;  // partial row of split 0
    const float2 a = lane < ns ? __ldcg(&ws.part_ml[row0 + static_cast<int64_t>(lane) * G]) : make_float2(-INFINITY, 0.f);
    const float2 c = lane + 32 < ns ? __ldcg(&ws.part_ml[row0 + static_cast<int64_t>(lane + 32) * G])
                                    : make_float2(-INFINITY, 0.f);
    float4 v[kCombineBatch];
#pragma unroll
    for (int i = 0; i < kCombineBatch; ++i)
      v[i] = i < ns ? __ldcg(po4 + (row0 + static_cast<int64_t>(i) * G) * (kHeadDim / 4) + lane)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    float M = fmaxf(a.x, c.x);
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float w = (M != -INFINITY && a.x != -INFINITY) ? ex2(a.x - M) : 0.f;
    const float w2 = (M != -INFINITY && c.x != -INFINITY) ? ex2(c.x - M) : 0.f;
    float L = w * a.y + w2 * c.y;
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < ns; s0 += kCombineBatch) {
      if (s0 > 0) {
#pragma unroll
        for (int i = 0; i < kCombineBatch; ++i)
          v[i] = s0 + i < ns ? __ldcg(po4 + (row0 + static_cast<int64_t>(s0 + i) * G) * (kHeadDim / 4) + lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < kCombineBatch; ++i) {
        const float wi = __shfl_sync(0xffffffffu, s0 + i < 32 ? w : w2, (s0 + i) & 31);
        if (s0 + i < ns) {
          acc.x += wi * v[i].x;
          acc.y += wi * v[i].y;
          acc.z += wi * v[i].z;
          acc.w += wi * v[i].w;
        }
      }
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    const int b = sp.x / Hkv, h = sp.x % Hkv;
    T* dst = out + static_cast<int64_t>(b) * out_stride + (static_cast<int64_t>(h) * G + n) * kHeadDim + lane * 4;
    dst[0] = from_float<T>(acc.x * inv);
    dst[1] = from_float<T>(acc.y * inv);
    dst[2] = from_float<T>(acc.z * inv);
    dst[3] = from_float<T>(acc.w * inv);
    if (item + n_warps < n_items) sp = ws.split_pairs[(item + n_warps) / G];
  }
}

// ---------------------------------------------------------------------------------------
// Host side: tensor maps, launch configuration.

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 5-D view of one of the K or V caches: (dim-lo 64, token 16, dim-hi D/64, head Hkv, block N).
// Token comes before dim-hi and head so that the 16 token rows of one (head, dim-half) sit in
// consecutive 128-byte shared-memory rows, which the 128-byte swizzle spreads over all banks.
int encode_kv_map(CUtensorMap* map, const void* base, int dtype, int Hkv, int64_t block_stride, int64_t num_blocks) {
  auto fn = get_encode_fn();
  if (!fn) return set_error(AEG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t es = 2;
  cuuint64_t dims[5] = {64, 16, static_cast<cuuint64_t>(kHalves), static_cast<cuuint64_t>(Hkv),
                        static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(Hkv) * kHeadDim * es, 64 * es, kHeadDim * es,
                           static_cast<cuuint64_t>(block_stride) * es};
  cuuint32_t box[5] = {64, 16, static_cast<cuuint32_t>(kHalves), 1, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dtype == AEG_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AEG_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return AEG_OK;
}

// Resident CTAs per SM of the attention kernel (occupancy API, cached per device; the first
// call on a device also raises the kernel's dynamic shared-memory limit).
template <typename T, int NT>
int attn_ctas_per_sm() {
  auto kern = decode_attn_kernel<T, NT>;
  constexpr size_t smem = AttnSmem<NT>::kDynamic;
  constexpr int kMaxDevices = 64;
  static int cache[kMaxDevices] = {0};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem) != cudaSuccess || n <= 0)
      n = -1;
    cache[dev] = n;
  }
  return cache[dev];
}

int ctas_per_sm(int dtype, int nt) {
  if (dtype == AEG_DTYPE_BF16) return nt == 1 ? attn_ctas_per_sm<__nv_bfloat16, 1>() : attn_ctas_per_sm<__nv_bfloat16, 2>();
  return nt == 1 ? attn_ctas_per_sm<__half, 1>() : attn_ctas_per_sm<__half, 2>();
}

cudaLaunchAttribute pdl_attr() {
  cudaLaunchAttribute a{};
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  return a;
}

template <typename T, int NT>
int launch_attn_t(const CUtensorMap& km, const CUtensorMap& vm, const AttnParams& prm, cudaStream_t stream) {
  const int per_sm = attn_ctas_per_sm<T, NT>();
  if (per_sm < 1) {
    (void)cudaGetLastError();
    return set_error(AEG_ERR_CUDA, "decode attention kernel cannot be configured on this device");
  }
  cudaLaunchAttribute attr[1] = {pdl_attr()};
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms() * per_sm));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = AttnSmem<NT>::kDynamic;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AEG_CHECK_CUDA(cudaLaunchKernelEx(&cfg, decode_attn_kernel<T, NT>, km, vm, prm));

  cudaLaunchConfig_t cc{};
  cc.gridDim = dim3(static_cast<unsigned>(num_sms() * 4));
  cc.blockDim = dim3(kCombineThreads);
  cc.dynamicSmemBytes = 0;
  cc.stream = stream;
  cc.attrs = attr;
  cc.numAttrs = 1;
  AEG_CHECK_CUDA(cudaLaunchKernelEx(&cc, decode_combine_kernel<T>, prm.out, prm.out_stride, prm.G, prm.Hkv, prm.ws));
  return AEG_OK;
}

int validate_shape(int B, int Hq, int Hkv, int D, int table_stride) {
  AEG_CHECK_ARG(B >= 0, "decode: negative batch");
  AEG_CHECK_ARG(Hkv > 0 && Hq > 0 && Hq % Hkv == 0, "decode: Hq (%d) must be a positive multiple of Hkv (%d)", Hq, Hkv);
  AEG_CHECK_ARG(Hq / Hkv <= 16, "decode: GQA group Hq/Hkv = %d exceeds 16", Hq / Hkv);
  if (D != kHeadDim) return set_error(AEG_ERR_UNSUPPORTED, "decode: head_dim %d not supported (only 128)", D);
  AEG_CHECK_ARG(table_stride > 0, "decode: block-table stride must be positive");
  AEG_CHECK_ARG(static_cast<int64_t>(B) * Hkv < (1 << 30), "decode: batch too large");
  return AEG_OK;
}

int decode_common(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_new,
                  int64_t k_new_stride, const void* v_new, int64_t v_new_stride, void* k_cache, void* v_cache,
                  int64_t block_stride, int64_t num_blocks, const int32_t* block_tables, int table_stride,
                  const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale, int dtype, void* workspace,
                  size_t workspace_bytes, void* stream, bool fuse, const WsLayout* layout = nullptr) {
  int st = validate_shape(B, Hq, Hkv, D, table_stride);
  if (st != AEG_OK) return st;
  if (B == 0) return AEG_OK;
  AEG_CHECK_ARG(dtype == AEG_DTYPE_FP16 || dtype == AEG_DTYPE_BF16, "decode: dtype %d is not fp16/bf16", dtype);
  AEG_CHECK_ARG(out && q && k_cache && v_cache && block_tables && seq_lens, "decode: null pointer");
  AEG_CHECK_ARG(workspace != nullptr && aligned(workspace, 256), "decode: workspace must be 256-byte aligned");
  const WsLayout L = layout ? *layout : ws_layout(B, Hq, Hkv, D);
  AEG_CHECK_ARG(workspace_bytes >= L.total, "decode: workspace of %zu bytes, need %zu", workspace_bytes, L.total);
  AEG_CHECK_ARG(num_blocks > 0 && num_blocks <= 0x7fffffffLL, "decode: num_blocks %lld out of range", (long long)num_blocks);
  AEG_CHECK_ARG(aligned(k_cache, 16) && aligned(v_cache, 16), "decode: K/V cache bases must be 16-byte aligned");
  AEG_CHECK_ARG(block_stride % 8 == 0 && block_stride >= int64_t(16) * Hkv * D,
                "decode: block stride %lld must be a multiple of 8 elements and >= 16*Hkv*D", (long long)block_stride);
  AEG_CHECK_ARG(q_stride >= int64_t(Hq) * D && out_stride >= int64_t(Hq) * D, "decode: q/out token stride < Hq*D");
  AEG_CHECK_ARG(aligned(q, 4) && q_stride % 2 == 0, "decode: q must be 4-byte aligned with an even token stride");
  AEG_CHECK_ARG(aligned(out, 2), "decode: out must be 2-byte aligned");
  AEG_CHECK_ARG(aligned(block_tables, 4) && aligned(seq_lens, 4), "decode: int32 arrays must be aligned");
  if (fuse) {
    AEG_CHECK_ARG(k_new && v_new, "decode_layer: null key/value pointer");
    AEG_CHECK_ARG(k_new_stride >= int64_t(Hkv) * D && v_new_stride >= int64_t(Hkv) * D,
                  "decode_layer: key/value token stride < Hkv*D");
    AEG_CHECK_ARG(aligned(k_new, 4) && aligned(v_new, 4) && k_new_stride % 2 == 0 && v_new_stride % 2 == 0,
                  "decode_layer: key/value must be 4-byte aligned with even token strides");
  }

  CUtensorMap km, vm;
  st = encode_kv_map(&km, k_cache, dtype, Hkv, block_stride, num_blocks);
  if (st != AEG_OK) return st;
  st = encode_kv_map(&vm, v_cache, dtype, Hkv, block_stride, num_blocks);
  if (st != AEG_OK) return st;

  AttnParams prm{};
  prm.out = out;
  prm.out_stride = out_stride;
  prm.q = q;
  prm.q_stride = q_stride;
  prm.tables = block_tables;
  prm.table_stride = table_stride;
  prm.seq_lens = seq_lens;
  prm.G = Hq / Hkv;
  prm.Hkv = Hkv;
  prm.num_pairs = B * Hkv;
  prm.max_units = L.max_units;
  prm.num_blocks = num_blocks;
  prm.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);  // log2(e)
  prm.q_bulk = (aligned(q, 16) && q_stride % 8 == 0) ? 1 : 0;
  prm.fuse_write = fuse ? 1 : 0;
  prm.k_new = k_new;
  prm.v_new = v_new;
  prm.k_new_stride = k_new_stride;
  prm.v_new_stride = v_new_stride;
  prm.k_cache = k_cache;
  prm.v_cache = v_cache;
  prm.block_stride = block_stride;
  prm.ws = ws_ptrs(workspace, L);
  const int nt = prm.G <= 8 ? 1 : 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AEG_DTYPE_BF16)
    return nt == 1 ? launch_attn_t<__nv_bfloat16, 1>(km, vm, prm, s) : launch_attn_t<__nv_bfloat16, 2>(km, vm, prm, s);
  return nt == 1 ? launch_attn_t<__half, 1>(km, vm, prm, s) : launch_attn_t<__half, 2>(km, vm, prm, s);
}

// ---------------------------------------------------------------------------------------
// Allocation-free decode attention (aeg_paged_attn_decode_noalloc).
//
// Some callers cannot hand this library a workspace and must not make it allocate one: a host
// that binds only the C ABI and owns no device allocator, code that runs inside an allocator
// or memory-pool callback (where allocating again would recurse into the allocator), and
// serving loops whose device memory has all been handed to the KV-block pool up front, so a
// cudaMalloc there would fail or evict cache blocks. For them this entry plans and runs the
// attention in a fixed scratch area held in this module's own static device memory. The
// driver reserves it, once per device, when it loads the module; the call itself allocates
// nothing.
//
// Limits and rules of use:
//   * The scratch holds kNoAllocScratchBytes (32 MiB) per device. Its layout is the workspace
//     layout with room for the units the plan actually makes (target + B*Hkv, where the target
//     is the one aeg_decode_plan uses by default), so the need grows with B*Hkv and the GQA
//     group: about 9.6 MB for 64 sequences x 4 KV heads x 7 query heads each. A call that
//     would need more is rejected with AEG_ERR_INVALID_ARGUMENT before anything is enqueued.
//   * Nothing in the scratch has to start at zero for the first call: the plan kernel that
//     every call enqueues writes the whole header, including the work and exit counters that
//     the attention kernel needs at zero, and the last warp of the attention kernel sets them
//     back to zero. (Static device memory also starts zeroed when the module is loaded.)
//   * One scratch per device means calls on one device must not overlap: two calls in flight
//     at once on different streams race on the plan, the counters and the partials. Issue
//     them on one stream, or order the streams.
//   * The first call on a device does one-time set-up with that device current: it looks up
//     the scratch address (cudaGetSymbolAddress, which may load the module) and configures
//     the attention kernel's shared-memory limit. Make that first call before any stream
//     capture begins.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of the current device's scratch, looked up once per device.
int noalloc_scratch(void** ptr) {
  int dev = 0;
  AEG_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(AEG_ERR_UNSUPPORTED, "decode_noalloc: device ordinal %d >= %d", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return set_error(AEG_ERR_CUDA, "decode_noalloc: cudaGetSymbolAddress of the scratch failed on device %d: %s", dev,
                       cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = p;
  }
  *ptr = g_noalloc_ptr[dev];
  return AEG_OK;
}

// The workspace layout with room for max_units units (the regular layout reserves
// kMaxTargetUnits + B*Hkv, far more than the default plan makes).
WsLayout noalloc_layout(int B, int Hq, int Hkv, int D, int max_units) {
  WsLayout w{};
  const int G = Hq / Hkv;
  const int64_t P = int64_t(B) * Hkv;
  w.max_units = max_units;
  size_t off = 256;
  w.split_pairs = off;
  off = align256(off + sizeof(int4) * P);
  w.units = off;
  off = align256(off + 2 * sizeof(int4) * size_t(max_units));
  w.part_ml = off;
  off = align256(off + sizeof(float2) * size_t(max_units) * G);
  w.part_o = off;
  off = align256(off + sizeof(float) * size_t(max_units) * G * D);
  w.total = off;
  return w;
}

}  // namespace

uint32_t deverr_read_and_clear_attn(cudaStream_t s, cudaError_t* err) {
  uint32_t v = 0, zero = 0;
  *err = cudaMemcpyFromSymbolAsync(&v, g_deverr_attn, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  if (*err == cudaSuccess) *err = cudaMemcpyToSymbolAsync(g_deverr_attn, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  return v;
}

}  // namespace aeg

extern "C" {

size_t aeg_decode_workspace_size(int B, int Hq, int Hkv, int D) {
  if (B < 0 || Hkv <= 0 || Hq <= 0 || Hq % Hkv != 0 || D <= 0) return 0;
  return aeg::ws_layout(B, Hq, Hkv, D).total;
}

int aeg_decode_plan(void* workspace, size_t workspace_bytes, const int32_t* block_tables, int table_stride,
                    const int32_t* seq_lens, int B, int Hq, int Hkv, int D, void* stream) {
  int st = aeg::validate_shape(B, Hq, Hkv, D, table_stride);
  if (st != AEG_OK) return st;
  AEG_CHECK_ARG(workspace != nullptr && aeg::aligned(workspace, 256), "decode_plan: workspace must be 256-byte aligned");
  const aeg::WsLayout L = aeg::ws_layout(B, Hq, Hkv, D);
  AEG_CHECK_ARG(workspace_bytes >= L.total, "decode_plan: workspace of %zu bytes, need %zu", workspace_bytes, L.total);
  AEG_CHECK_ARG(B == 0 || (seq_lens != nullptr && block_tables != nullptr), "decode_plan: seq_lens/block_tables is NULL");
  AEG_CHECK_ARG(aeg::aligned(seq_lens, 4) && aeg::aligned(block_tables, 4), "decode_plan: int32 arrays must be aligned");
  // Balanced unit count: a few units per worker warp so that the dynamic scheduler can even
  // out the tail. AEG_DECODE_UNITS_PER_WARP overrides the factor (tuning experiments).
  int per_warp = 2;
  if (const char* e = std::getenv("AEG_DECODE_UNITS_PER_WARP")) {
    const int k = std::atoi(e);
    if (k > 0) per_warp = k;
  }
  const int per_sm = aeg::ctas_per_sm(AEG_DTYPE_FP16, (Hq / Hkv) <= 8 ? 1 : 2);
  long long target = static_cast<long long>(aeg::num_sms()) * (per_sm > 0 ? per_sm : 1) * aeg::kWarps * per_warp;
  if (target > aeg::kMaxTargetUnits) target = aeg::kMaxTargetUnits;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  aeg::WsPtrs w = aeg::ws_ptrs(workspace, L);
  aeg::decode_plan_kernel<<<1, aeg::kPlanThreads, 0, s>>>(seq_lens, block_tables, B, Hkv, table_stride,
                                                          static_cast<int>(target), w);
  AEG_CHECK_LAUNCH("decode_plan");
  return AEG_OK;
}

int aeg_paged_attn_decode(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_cache,
                          const void* v_cache, int64_t block_stride, int64_t num_blocks, const int32_t* block_tables,
                          int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale,
                          int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  return aeg::decode_common(out, out_stride, q, q_stride, nullptr, 0, nullptr, 0, const_cast<void*>(k_cache),
                            const_cast<void*>(v_cache), block_stride, num_blocks, block_tables, table_stride, seq_lens, B,
                            Hq, Hkv, D, scale, dtype, workspace, workspace_bytes, stream, false);
}

int aeg_decode_layer(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* key_new,
                     int64_t key_stride, const void* value_new, int64_t value_stride, void* k_cache, void* v_cache,
                     int64_t block_stride, int64_t num_blocks, const int32_t* block_tables, int table_stride,
                     const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale, int dtype, void* workspace,
                     size_t workspace_bytes, void* stream) {
  return aeg::decode_common(out, out_stride, q, q_stride, key_new, key_stride, value_new, value_stride, k_cache, v_cache,
                            block_stride, num_blocks, block_tables, table_stride, seq_lens, B, Hq, Hkv, D, scale, dtype,
                            workspace, workspace_bytes, stream, true);
}

// Plan + attention + split merge in the static per-device scratch (no counterpart in the
// reference; see the allocation-free section above for limits and rules of use).
int aeg_paged_attn_decode_noalloc(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_cache,
                                  const void* v_cache, int64_t block_stride, int64_t num_blocks,
                                  const int32_t* block_tables, int table_stride, const int32_t* seq_lens, int B, int Hq,
                                  int Hkv, int D, float scale, int dtype, void* stream) {
  int st = aeg::validate_shape(B, Hq, Hkv, D, table_stride);
  if (st != AEG_OK) return st;
  if (B == 0) return AEG_OK;
  AEG_CHECK_ARG(dtype == AEG_DTYPE_FP16 || dtype == AEG_DTYPE_BF16, "decode_noalloc: dtype %d is not fp16/bf16", dtype);
  AEG_CHECK_ARG(out && q && k_cache && v_cache && block_tables && seq_lens, "decode_noalloc: null pointer");
  AEG_CHECK_ARG(aeg::aligned(seq_lens, 4) && aeg::aligned(block_tables, 4), "decode_noalloc: int32 arrays must be aligned");
  const int per_sm = aeg::ctas_per_sm(AEG_DTYPE_FP16, (Hq / Hkv) <= 8 ? 1 : 2);
  long long target = static_cast<long long>(aeg::num_sms()) * (per_sm > 0 ? per_sm : 1) * aeg::kWarps * 2;
  if (target > aeg::kMaxTargetUnits) target = aeg::kMaxTargetUnits;
  const aeg::WsLayout L =
      aeg::noalloc_layout(B, Hq, Hkv, D, static_cast<int>(target + static_cast<long long>(B) * Hkv));
  AEG_CHECK_ARG(L.total <= aeg::kNoAllocScratchBytes,
                "decode_noalloc: B=%d, Hq=%d, Hkv=%d needs %zu bytes of scratch, more than the %zu bytes of the "
                "static scratch; use aeg_paged_attn_decode with a caller-owned workspace",
                B, Hq, Hkv, L.total, aeg::kNoAllocScratchBytes);
  void* scratch = nullptr;
  st = aeg::noalloc_scratch(&scratch);
  if (st != AEG_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  aeg::decode_plan_kernel<<<1, aeg::kPlanThreads, 0, s>>>(seq_lens, block_tables, B, Hkv, table_stride,
                                                          static_cast<int>(target), aeg::ws_ptrs(scratch, L));
  AEG_CHECK_LAUNCH("decode_plan (noalloc)");
  return aeg::decode_common(out, out_stride, q, q_stride, nullptr, 0, nullptr, 0, const_cast<void*>(k_cache),
                            const_cast<void*>(v_cache), block_stride, num_blocks, block_tables, table_stride, seq_lens, B,
                            Hq, Hkv, D, scale, dtype, scratch, aeg::kNoAllocScratchBytes, stream, false, &L);
}

}  // extern "C"
