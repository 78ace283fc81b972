// Paged decode attention over Aegaeon's block-table KV cache, written for sm_100a.
//
// Semantics: the decode call of the vLLM 0.5.1 FlashAttention backend that the reference runs
// per layer (flash_attn_with_kvcache(q[:, None], K_l, V_l, block_table, cache_seqlens, scale,
// causal=True) reached from aegaeon/aegaeon/worker.py:517-523, metadata from worker.py:554-713).
// One query token per sequence, so every cached key j < seq_len is visible; query head h reads
// KV head h / (Hq / Hkv).
//
// Design (memory-bound: every K/V byte is read exactly once per layer call):
//   * Work item = one 16-token block of one (sequence b, KV head h) pair. A plan kernel, run
//     once per decode step, cuts the batch's items (in pair order) into W contiguous ranges of
//     equal size, one per worker warp of the attention grid (W = 8 warps x one CTA per SM).
//     A worker's range is a list of units (pieces of pairs); a pair cut by a worker start is
//     "split", and its units write partials. A unit record carries the pair, its block range,
//     its partial slot, the sequence length and its first three block ids.
//   * Every warp works through its own range with no scheduling traffic: its unit records sit
//     in its lanes (one load for the first, one coalesced load for the next 31), so moving on
//     to the next unit needs no global round trip. It streams each (block, head) K and V tile
//     (16 tokens x 128 dims, 4 KiB each) into its own kStages-deep shared-memory ring with 5-D
//     bulk-tensor TMA loads (128-byte swizzle, evict-first L2 policy) completing on
//     mbarriers, kStages tiles ahead of the compute, across unit boundaries. The next unit's
//     query rows are bulk-copied while the current unit is computed.
//   * Per block the warp computes S^T = K Q^T with mma.sync m16n8k16 (16 tokens x 8 query
//     heads of the GQA group; K fragments by ldmatrix from the swizzled tile), an fp32 online
//     softmax in the exp2 domain with quad shuffles, transposes P in registers with movmatrix
//     and accumulates O^T += V^T P^T (V fragments by ldmatrix.trans). For bf16, P enters as a
//     bf16 value plus its bf16 rounding residue (two MMAs) so that P V keeps ~16 mantissa bits.
//   * A whole pair's unit writes the output rows; a split unit writes an fp32 partial (O scaled
//     by 2^-max, max, sum). When its range is done each worker warp stamps its own flag (its own
//     cache line) with the launch's epoch by a release store. Every warp stamps its flag once
//     per launch, so all flags hold the same value between launches (the plan zeroes them) and a
//     warp takes the epoch from its own flag, with no end-of-launch counter. Then all warps merge
//     the split pairs: the plan spreads the merge items evenly over the warps, and an item waits
//     only for the flags of the warps that computed its pair's pieces (one CTA per SM: all CTAs
//     are resident together; a CTA-wide publication made every merge wait for the slowest warp of
//     each producing CTA, ~1 us). A
//     merge item covers 4 query heads of a pair with up to 4 pieces, one head of a pair with
//     up to 16 (in 4 lane groups), or a dimension chunk of one head beyond that, so that a lane
//     folds at most 4 (16) pieces loaded in one round trip. Measured and rejected: signalling
//     every split (fence + counter per split, the last one merges) cost ~2.5 us per split under
//     full HBM load; a grid-wide barrier before the merge made every item wait for the slowest
//     CTA; merging each pair in the CTA that computed its last piece piled the long and the
//     short-sequence pairs onto a few CTAs; a dynamic unit queue left ~2 us gaps at every unit
//     change; polling packed flags with short sleeps slowed the flag stores themselves.
//   * Fused form (aeg_decode_layer): the warp that reads a sequence's newest block writes the
//     new token's K/V row of its head into the cache and patches it into the tile.
//   * Every wait is bounded (2 s); a timeout raises AEG_DEVERR_WAIT_TIMEOUT and the warp
//     drains instead of hanging.
#include "aeg_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <mutex>
#include <unordered_set>
#include <type_traits>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_attn = 0;

constexpr int kHeadDim = 128;
constexpr int kHalves = kHeadDim / 64;  // 128-byte rows per (token, head)
constexpr int kBlockTokens = 16;
constexpr int kMaxWarps = 4096;         // worker warps of one launch the workspace is sized for
constexpr int kPlanThreads = 256;
constexpr int kUnitCost = 2;           // plan cost of starting a pair, in blocks (query load, epilogue)
constexpr int kPlanLongUnits = 4;       // a pair with more units has them written by the whole plan CTA
constexpr int kPlanLongPairs = 512;     // capacity of the plan's list of such pairs
constexpr int kPlanCachedSeqs = 4096;   // sequences whose block counts the plan keeps in smem
constexpr uint64_t kWaitLimitNs = 2000000000ull;

constexpr int kWarps = 8;               // independent workers per CTA (one CTA per SM)
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 3;              // per-warp ring depth
constexpr int kBoxBytes = kHalves * kBlockTokens * 128;  // one (block, head) K or V tile: 4 KiB
constexpr int kStageBytes = 2 * kBoxBytes;

// Header words of the workspace.
constexpr int kHdrItems = 0, kHdrWarps = 1, kHdrUnits = 2, kHdrSplitPairs = 3, kHdrSlots = 4,
              kHdrMergeItems = 5;
constexpr int kFlagStride = 32;  // int32 words between worker-warp flags: one 128-byte line each
constexpr int kMergeBatch = 16;      // pieces a lane loads per round trip in the split merge
constexpr int kMergeLaneGroups = 4;  // lane groups of a small merge item (heads or piece groups)
constexpr int kMergeHeadBatch = 4;   // pieces a lane of a small merge item folds per round trip

// ---------------------------------------------------------------------------------------
// Workspace layout (all offsets 256-byte aligned):
//   header      : int32[64]  {items, warps, units, split pairs, partial slots, merge items}
//   warp_rec    : int4[3 * (max_warps + 1)]  per worker warp w: {first unit, 0, 0, 0} and a copy of
//                            its first unit's record (one load starts a warp); entry `warps`
//                            holds the end of the unit list
//   split_pairs : int4[P]    {pair, first partial slot, nsplit | shape << 16, first warp |
//                            warps << 16} of every (sequence, head) cut across warps (nsplit
//                            >= 2) and {pair, 0, shape << 16, 0} of every empty one; its merge
//                            is merge_items(shape) items, which wait for the worker warps that
//                            computed its pieces
//   warp_flag   : int32[max_warps * kFlagStride] per worker warp (one cache line each): the
//                            number of launches with this plan whose partials it has published
//   merge_rec   : int4[max_warps]  per warp: {split-pair entry, item within it, items, 0}, its
//                            share of the merge items (balanced like the blocks)
//   units       : int4[2 * max_units]  {pair, j0, j1, partial slot or -1},
//                                      {seq_len, block id of items 0, 1, 2}
//   part_ml     : float2[max_slots * G]        (max in log2 units, sum) per query head
//   part_o      : float [max_slots * G * D]    partial outputs, scaled by 2^-max
struct WsLayout {
  size_t warp_rec, split_pairs, warp_flag, merge_rec, units, part_ml, part_o, total;
  int max_warps, max_units, max_slots;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Units: one per non-empty pair plus one per cut (a worker's range starting inside a pair), so
// at most P + warps. Partial slots: only units of cut pairs have one, at most 2 * warps.
WsLayout layout_for(int B, int Hq, int Hkv, int D, int max_warps) {
  WsLayout w{};
  const int G = Hq / Hkv;
  const int64_t P = int64_t(B) * Hkv;
  w.max_warps = max_warps;
  w.max_units = static_cast<int>(P + max_warps);
  w.max_slots = 2 * max_warps;
  size_t off = 256;
  w.warp_rec = off;
  off = align256(off + 3 * sizeof(int4) * size_t(max_warps + 1));
  w.split_pairs = off;
  off = align256(off + sizeof(int4) * P);
  w.warp_flag = off;
  off = align256(off + sizeof(int) * size_t(max_warps) * kFlagStride);
  w.merge_rec = off;
  off = align256(off + sizeof(int4) * size_t(max_warps));
  w.units = off;
  off = align256(off + 2 * sizeof(int4) * size_t(w.max_units));
  w.part_ml = off;
  off = align256(off + sizeof(float2) * size_t(w.max_slots) * G);
  w.part_o = off;
  off = align256(off + sizeof(float) * size_t(w.max_slots) * G * D);
  w.total = off;
  return w;
}

WsLayout ws_layout(int B, int Hq, int Hkv, int D) { return layout_for(B, Hq, Hkv, D, kMaxWarps); }

struct WsPtrs {
  int* header;
  int4* warp_rec;
  int4* split_pairs;
  int* warp_flag;
  int4* merge_rec;
  int4* units;
  float2* part_ml;
  float* part_o;
};

inline WsPtrs ws_ptrs(void* ws, const WsLayout& L) {
  char* b = static_cast<char*>(ws);
  return WsPtrs{reinterpret_cast<int*>(b), reinterpret_cast<int4*>(b + L.warp_rec),
                reinterpret_cast<int4*>(b + L.split_pairs), reinterpret_cast<int*>(b + L.warp_flag),
                reinterpret_cast<int4*>(b + L.merge_rec),
                reinterpret_cast<int4*>(b + L.units),
                reinterpret_cast<float2*>(b + L.part_ml), reinterpret_cast<float*>(b + L.part_o)};
}

// ---------------------------------------------------------------------------------------
// Plan kernel (one CTA). The (pair, block) items of the batch, in pair order, each non-empty
// pair preceded by kUnitCost virtual items (the cost of starting a pair), form a cost axis of
// I positions, cut into Wp = min(W, I) contiguous ranges of equal size (up to one position),
// one per worker warp: worker w < Wp starts at position floor(w * I / Wp), workers from Wp on
// get nothing. Units are the pieces of pairs' blocks between pair ends and worker starts; a
// worker starting on a pair's virtual positions begins with the pair's first block.

__device__ __forceinline__ int seq_blocks(const int* seq_lens, int b, int cap, bool report) {
  int n = seq_lens[b];
  if (n < 0 || n > cap) {
    if (report) atomicOr(&g_deverr_attn, AEG_DEVERR_SEQ_LEN_RANGE);
    n = n < 0 ? 0 : cap;
  }
  return (n + kBlockTokens - 1) / kBlockTokens;
}

// Division of non-negative 64-bit values below 2^63 by a divisor fixed for the whole plan:
// a multiply-high by m = floor((2^64 - 1) / d) and one correction step (Granlund and
// Montgomery, "Division by invariant integers using multiplication", 1994). m * d >= 2^64 - d,
// so n * m / 2^64 > n / d - 1/2 for n < 2^63 and the estimate is floor(n / d) or one less.
struct InvariantDiv {
  unsigned long long d, m;
  __device__ explicit InvariantDiv(long long divisor)
      : d(static_cast<unsigned long long>(divisor)), m(divisor > 0 ? ~0ULL / d : 0ULL) {}
  __device__ __forceinline__ long long operator()(long long n) const {
    const unsigned long long un = static_cast<unsigned long long>(n);
    unsigned long long q = __umul64hi(un, m);
    if (un - q * d >= d) ++q;
    return static_cast<long long>(q);
  }
};

// Products stay below 2^63: I <= kMaxItems and w, W <= kMaxWarps.
constexpr long long kMaxItems = 1LL << 48;

// Cuts of a cost axis of I positions into W equal ranges: worker w starts at floor(w * I / W).
struct EqualCuts {
  long long I;
  int W;
  InvariantDiv by_w, by_i;
  __device__ EqualCuts(long long I_, int W_) : I(I_), W(W_), by_w(W_), by_i(I_) {}
  // First position of worker w.
  __device__ __forceinline__ long long start(long long w) const { return by_w(w * I); }
  // Number of workers whose first position is <= x (worker 0 starts at position 0).
  __device__ __forceinline__ long long le(long long x) const {
    if (x < 0) return 0;
    const long long c = by_i((x + 1) * W + I - 1);
    return c < W ? c : W;
  }
};

// Shape of a pair's merge (merge_small / merge_item): up to 4 pieces, an item covers the whole
// rows of 4 query heads (hg = 4); 5..kMergeBatch pieces, one query head (hg = 1); more pieces
// are cut into q dimension chunks of one head each, so that a lane loads at most kMergeBatch
// pieces. Encoded as q | hg << 8 in the split-pair entry.
__host__ __device__ __forceinline__ int merge_shape(int ns, int G) {
  if (ns <= kMergeLaneGroups) return 1 | (kMergeLaneGroups << 8);  // heads mode
  if (ns <= kMergeBatch) return 1 | (1 << 8);                        // pieces mode
  int q = 1;
  while (q < 32 && ns > q * kMergeBatch) q *= 2;
  return q | (1 << 8);
}

// Merge items of a pair with merge shape `shape`.
__host__ __device__ __forceinline__ int merge_items(int shape, int G) {
  const int q = shape & 0xff, hg = shape >> 8;
  return ((G + hg - 1) / hg) * q;
}

// Block-wide exclusive scans of one value per thread; also return the total.
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

__device__ __forceinline__ long long block_excl_scan64(long long v, long long* s_warp, long long& total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  long long incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const long long t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) s_warp[wid] = incl;
  __syncthreads();
  long long off = 0;
  total = 0;
  for (int i = 0; i < kPlanThreads / 32; ++i) {
    if (i < wid) off += s_warp[i];
    total += s_warp[i];
  }
  return off + incl - v;
}

__global__ void __launch_bounds__(kPlanThreads, 1)
decode_plan_kernel(const int* __restrict__ seq_lens, const int* __restrict__ tables, int B, int Hkv,
                   int G, int table_stride, int W, WsPtrs ws) {
  __shared__ long long s_red[kPlanThreads / 32];
  __shared__ int s_warp[kPlanThreads / 32];
  __shared__ int s_nb[kPlanCachedSeqs];  // blocks per sequence (first kPlanCachedSeqs sequences)
  __shared__ int4 s_long[kPlanLongPairs];         // {pair, first unit, cuts, first slot}
  __shared__ long long s_long_o[kPlanLongPairs];  // position of the pair's first block
  __shared__ int s_long_ofs[kPlanLongPairs + 1];  // prefix sums of the pairs' unit counts
  __shared__ int s_nlong;
  const int tid = threadIdx.x;
  if (tid == 0) s_nlong = 0;
  const int P = B * Hkv;
  const int cap = table_stride * kBlockTokens;
  const int per = (P + kPlanThreads - 1) / kPlanThreads;
  const int p0 = min(P, tid * per), p1 = min(P, p0 + per);

  for (int b = tid; b < B; b += kPlanThreads) {
    const int nb = seq_blocks(seq_lens, b, cap, true);
    if (b < kPlanCachedSeqs) s_nb[b] = nb;
  }
  __syncthreads();
  auto blocks_of = [&](int b) { return b < kPlanCachedSeqs ? s_nb[b] : seq_blocks(seq_lens, b, cap, false); };

  // Pass 1: items of this thread's pairs -> item offset of its first pair, total I.
  long long local = 0;
  for (int p = p0; p < p1; ++p) {
    const int nb = blocks_of(p / Hkv);
    local += nb > 0 ? nb + kUnitCost : 0;
  }
  long long I = 0;
  const long long o_t = block_excl_scan64(local, s_red, I);
  if (I > kMaxItems) {  // beyond any pool this plan can address: plan nothing, report it
    if (tid == 0) {
      atomicOr(&g_deverr_attn, AEG_DEVERR_SEQ_LEN_RANGE);
      ws.header[kHdrWarps] = W;
      ws.header[kHdrUnits] = 0;
      ws.header[kHdrSplitPairs] = 0;
    }
    for (int w = tid; w <= W; w += kPlanThreads) ws.warp_rec[3 * w] = make_int4(0, 0, 0, 0);
    for (int w = tid; w < W; w += kPlanThreads) ws.merge_rec[w] = make_int4(0, 0, 0, 0);
    for (int c = tid; c < W; c += kPlanThreads) ws.warp_flag[c * kFlagStride] = 0;
    return;
  }
  const int Wp = I < W ? static_cast<int>(I) : W;  // workers with items; their starts are distinct
  const EqualCuts wk(I, Wp);
  auto cuts = [&](long long o, int nb) {  // workers starting strictly inside the pair's items
    return static_cast<int>(wk.le(o + nb - 1) - wk.le(o));
  };

  // Pass 2: units, split-pair entries, partial slots and merge items of this thread's pairs.
  int n_units = 0, n_sp = 0, n_slots = 0;
  long long n_mi = 0;
  long long o = o_t;
  for (int p = p0; p < p1; ++p) {
    const int nb = blocks_of(p / Hkv);
    if (nb == 0) {
      ++n_sp;
      n_mi += merge_items(merge_shape(0, G), G);
      continue;
    }
    const int c = cuts(o + kUnitCost, nb);
    n_units += c + 1;
    if (c > 0) {
      ++n_sp;
      n_slots += c + 1;
      n_mi += merge_items(merge_shape(c + 1, G), G);
    }
    o += nb + kUnitCost;
  }
  int U = 0, S = 0, SL = 0;
  int u = block_excl_scan(n_units, s_warp, U);
  int sp = block_excl_scan(n_sp, s_warp, S);
  int slot = block_excl_scan(n_slots, s_warp, SL);
  long long MI = 0;
  long long mo = block_excl_scan64(n_mi, s_red, MI);
  const int Wm = MI < W ? static_cast<int>(MI) : W;  // warps with merge items
  const EqualCuts mk(MI, Wm);
  // Warps whose share of the merge items starts in [mo0, mo0 + n) get {entry, item within it,
  // items}; warp w's share is [floor(w * MI / Wm), floor((w + 1) * MI / Wm)).
  auto mark_merge = [&](int entry, long long mo0, int n) {
    const long long w_hi = mk.le(mo0 + n - 1);
    for (long long w = mk.le(mo0 - 1); w < w_hi; ++w) {
      const long long st = mk.start(w);
      const long long en = w + 1 < Wm ? mk.start(w + 1) : MI;
      ws.merge_rec[w] = make_int4(entry, static_cast<int>(st - mo0), static_cast<int>(en - st), 0);
    }
  };
  if (tid == 0) {
    ws.header[kHdrItems] = static_cast<int>(I < 0x7fffffffLL ? I : 0x7fffffffLL);
    ws.header[kHdrWarps] = W;
    ws.header[kHdrUnits] = U;
    ws.header[kHdrSplitPairs] = S;
    ws.header[kHdrSlots] = SL;
    ws.header[kHdrMergeItems] = static_cast<int>(MI < 0x7fffffffLL ? MI : 0x7fffffffLL);
  }
  for (int c = tid; c < W; c += kPlanThreads) ws.warp_flag[c * kFlagStride] = 0;
  for (int w = Wp + tid; w <= W; w += kPlanThreads) ws.warp_rec[3 * w] = make_int4(U, 0, 0, 0);  // empty ranges
  for (int w = Wm + tid; w < W; w += kPlanThreads) ws.merge_rec[w] = make_int4(S, 0, 0, 0);      // no merge items

  // Pass 3: write units, split-pair entries and the workers' first-unit records. Unit k of a
  // pair spans items [xa, xb) between the pair's ends and the worker starts inside it; the
  // workers starting at xa begin with it. Pairs with many units (long sequences) are queued and
  // their units written by all threads below, so that no thread writes dozens of them, each
  // behind a block-table load.
  auto emit_unit = [&](int p, long long o0, int nb, int c, int k, int u_idx, int slot_idx) {
    const int b = p / Hkv;
    const long long wc = wk.le(o0);  // first worker starting after item o0
    const long long xa = k == 0 ? o0 : wk.start(wc + k - 1);
    const long long xb = k == c ? o0 + nb : wk.start(wc + k);
    const int j0 = static_cast<int>(xa - o0), j1 = static_cast<int>(xb - o0);
    const int n = j1 - j0;
    const int* tb = tables + static_cast<int64_t>(b) * table_stride + j0;
    const int n_ctx = min(max(seq_lens[b], 0), cap);
    const int4 ra = make_int4(p, j0, j1, c > 0 ? slot_idx : -1);
    const int4 rb = make_int4(n_ctx, tb[0], n > 1 ? tb[1] : 0, n > 2 ? tb[2] : 0);
    ws.units[2 * u_idx] = ra;
    ws.units[2 * u_idx + 1] = rb;
    const long long w_hi = wk.le(xa);
    for (long long w = wk.le((k == 0 ? o0 - kUnitCost : xa) - 1); w < w_hi; ++w) {
      ws.warp_rec[3 * w] = make_int4(u_idx, 0, 0, 0);
      ws.warp_rec[3 * w + 1] = ra;
      ws.warp_rec[3 * w + 2] = rb;
    }
  };
  o = o_t;
  for (int p = p0; p < p1; ++p) {
    const int nb = blocks_of(p / Hkv);
    if (nb == 0) {
      const int shape = merge_shape(0, G), n_it = merge_items(shape, G);
      mark_merge(sp, mo, n_it);
      mo += n_it;
      ws.split_pairs[sp++] = make_int4(p, 0, shape << 16, 0);
      continue;
    }
    const long long ob = o + kUnitCost;  // position of the pair's first block
    const int c = cuts(ob, nb);
    if (c > 0) {
      const int shape = merge_shape(c + 1, G), n_it = merge_items(shape, G);
      mark_merge(sp, mo, n_it);
      mo += n_it;
      const int w0 = static_cast<int>(wk.le(ob) - 1);           // worker holding the first block
      const int w1 = static_cast<int>(wk.le(ob + nb - 1) - 1);  // and the last
      ws.split_pairs[sp++] = make_int4(p, slot, (c + 1) | (shape << 16), w0 | ((w1 - w0 + 1) << 16));
    }
    int queued = -1;
    if (c + 1 > kPlanLongUnits) {
      queued = atomicAdd(&s_nlong, 1);
      if (queued < kPlanLongPairs) {
        s_long[queued] = make_int4(p, u, c, slot);
        s_long_o[queued] = ob;
      }
    }
    if (queued < 0 || queued >= kPlanLongPairs)
      for (int k = 0; k <= c; ++k) emit_unit(p, ob, nb, c, k, u + k, slot + k);
    u += c + 1;
    if (c > 0) slot += c + 1;
    o = ob + nb;
  }
  __syncthreads();
  const int n_long = min(s_nlong, kPlanLongPairs);
  {
    static_assert(kPlanLongPairs == 2 * kPlanThreads, "two queued pairs per plan thread");
    const int i0 = 2 * tid;
    const int v0 = i0 < n_long ? s_long[i0].z + 1 : 0, v1 = i0 + 1 < n_long ? s_long[i0 + 1].z + 1 : 0;
    int total = 0;
    const int e0 = block_excl_scan(v0 + v1, s_warp, total);
    s_long_ofs[i0] = e0;
    s_long_ofs[i0 + 1] = e0 + v0;
    if (tid == 0) s_long_ofs[kPlanLongPairs] = total;
  }
  __syncthreads();
  const int n_long_units = s_long_ofs[kPlanLongPairs];
  for (int t = tid; t < n_long_units; t += kPlanThreads) {
    int lo = 0, hi = n_long;  // the queued pair whose units include t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (s_long_ofs[mid] <= t) lo = mid; else hi = mid;
    }
    const int4 L = s_long[lo];
    const int k = t - s_long_ofs[lo];
    emit_unit(L.x, s_long_o[lo], blocks_of(L.x / Hkv), L.z, k, L.y + k, L.w + k);
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
  int max_warps;  // capacities of the workspace lists
  int max_units;
  int max_slots;
  int64_t num_blocks;
  float scale_log2;
  int q_bulk;  // query rows are 16-byte aligned: stage them with bulk copies
  int plan_ready;   // the plan was complete before the preceding kernel started: read it early
  int prefetch_kv;  // the preceding kernel writes neither these cache blocks nor the tables
  // Fused cache write (decode_layer): the new token of sequence b (position seq_len - 1) is
  // written into the cache and patched into the tile that holds it.
  int fuse_write;
  // The preceding kernel may have written the newest position (seq_len - 1) of each sequence
  // (the decode cache write) and nothing else this launch reads: tiles may be requested early,
  // and each sequence's newest row is read again after the grid-dependency wait and patched in.
  int refresh_last;
  const void* k_new;
  const void* v_new;
  int64_t k_new_stride;  // token strides of k_new / v_new (elements)
  int64_t v_new_stride;
  void* k_cache;
  void* v_cache;
  int64_t block_stride;  // elements
  WsPtrs ws;
};

// Items (blocks) of a unit record, or 0 if the record is not consistent with this call's shape:
// a workspace that was not planned for this call is skipped and reported instead of steering
// loads out of bounds.
__device__ __forceinline__ int unit_items(const int4& a, const int4& b, const AttnParams& p) {
  const bool ok = a.x >= 0 && a.x < p.num_pairs && a.y >= 0 && a.y < a.z && a.z <= p.table_stride && a.w >= -1 &&
                  a.w < p.max_slots && b.x >= 0 && b.x <= p.table_stride * kBlockTokens &&
                  a.z * kBlockTokens < b.x + kBlockTokens;
  return ok ? a.z - a.y : 0;
}

__device__ __forceinline__ int4 shfl4(const int4& v, int src) {
  return make_int4(__shfl_sync(0xffffffffu, v.x, src), __shfl_sync(0xffffffffu, v.y, src),
                   __shfl_sync(0xffffffffu, v.z, src), __shfl_sync(0xffffffffu, v.w, src));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ float2 ld_cg_f2(const float2* ptr) {
  float2 r;
  asm volatile("ld.global.cg.v2.f32 {%0, %1}, [%2];" : "=f"(r.x), "=f"(r.y) : "l"(ptr));
  return r;
}
// Empty volatile statement that claims to rewrite a loaded pair: placed after a batch of loads,
// it keeps the compiler from moving the folds that use the values above later loads of the
// batch (which would serialise the round trips).
__device__ __forceinline__ void after_loads(float2& a, float4& b) {
  asm volatile("" : "+f"(a.x), "+f"(a.y), "+f"(b.x), "+f"(b.y), "+f"(b.z), "+f"(b.w));
}

__device__ __forceinline__ float4 ld_cg_f4(const float4* ptr) {
  float4 r;
  asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(ptr));
  return r;
}

// Item of a pair with at most kMergeBatch pieces (q == 1), 4 lane groups of 8 lanes; a lane
// owns float4 columns c, c + 8, c + 16, c + 24 of a 128-dim row.
//   * heads mode (hg == 4, up to 4 pieces): group g takes query head item * 4 + g and folds its
//     pieces in order. An empty pair (ns = 0) gets zero rows.
//   * pieces mode (hg == 1, 5..16 pieces): the item is query head `item`; group g folds pieces
//     g, g + 4, g + 8, g + 12 and the 4 groups are combined by xor shuffles.
// Either way a lane folds at most 4 pieces, whose 16 row loads share one round trip.

template <typename T, typename WriteRow>
__device__ __forceinline__ void merge_small(const AttnParams& p, const int4& e, int item, int lane, bool by_pieces,
                                            WriteRow& write_row) {
  constexpr int kLanes = 32 / kMergeLaneGroups;  // lanes per group
  constexpr int kCols = kMergeLaneGroups;        // float4 columns per lane
  const int G = p.G, ns = e.z & 0xffff;
  const int grp = lane / kLanes, c = lane % kLanes;
  const int n = by_pieces ? item : item * kMergeLaneGroups + grp;
  const int p0 = by_pieces ? grp : 0, pstep = by_pieces ? kMergeLaneGroups : 1;
  const int mine = n >= G ? 0 : (by_pieces ? (ns - grp + kMergeLaneGroups - 1) / kMergeLaneGroups : ns);
  const float4* po4 = reinterpret_cast<const float4*>(p.ws.part_o);
  float M = -INFINITY, L = 0.f;
  float4 acc[kCols];
#pragma unroll
  for (int k = 0; k < kCols; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i0 = 0; i0 < mine; i0 += kMergeHeadBatch) {
    float2 ml[kMergeHeadBatch];
    float4 v[kMergeHeadBatch][kCols];
    const int cnt = min(kMergeHeadBatch, mine - i0);
#pragma unroll
    for (int i = 0; i < kMergeHeadBatch; ++i) {
      if (i >= cnt) break;
      const int64_t row = static_cast<int64_t>(e.y + p0 + (i0 + i) * pstep) * G + n;
      ml[i] = ld_cg_f2(&p.ws.part_ml[row]);
#pragma unroll
      for (int k = 0; k < kCols; ++k) v[i][k] = ld_cg_f4(po4 + row * (kHeadDim / 4) + c + k * kLanes);
    }
#pragma unroll
    for (int i = 0; i < kMergeHeadBatch; ++i) {
      if (i >= cnt) break;
#pragma unroll
      for (int k = 0; k < kCols; ++k) after_loads(ml[i], v[i][k]);
    }
#pragma unroll
    for (int i = 0; i < kMergeHeadBatch; ++i) {
      if (i >= cnt) break;
      if (ml[i].x != -INFINITY) {
        const float Mn = fmaxf(M, ml[i].x);
        const float r = M != -INFINITY ? ex2(M - Mn) : 0.f;
        const float w = ex2(ml[i].x - Mn);
#pragma unroll
        for (int k = 0; k < kCols; ++k) {
          acc[k].x = acc[k].x * r + w * v[i][k].x;
          acc[k].y = acc[k].y * r + w * v[i][k].y;
          acc[k].z = acc[k].z * r + w * v[i][k].z;
          acc[k].w = acc[k].w * r + w * v[i][k].w;
        }
        L = L * r + w * ml[i].y;
        M = Mn;
      }
    }
  }
  if (by_pieces) {
#pragma unroll
    for (int off = kLanes; off < 32; off <<= 1) {
      const float Mo = __shfl_xor_sync(0xffffffffu, M, off);
      const float Lo = __shfl_xor_sync(0xffffffffu, L, off);
      const float Mn = fmaxf(M, Mo);
      const float r1 = M != -INFINITY ? ex2(M - Mn) : 0.f;
      const float r2 = Mo != -INFINITY ? ex2(Mo - Mn) : 0.f;
#pragma unroll
      for (int k = 0; k < kCols; ++k) {
        float4 ao;
        ao.x = __shfl_xor_sync(0xffffffffu, acc[k].x, off);
        ao.y = __shfl_xor_sync(0xffffffffu, acc[k].y, off);
        ao.z = __shfl_xor_sync(0xffffffffu, acc[k].z, off);
        ao.w = __shfl_xor_sync(0xffffffffu, acc[k].w, off);
        acc[k].x = acc[k].x * r1 + ao.x * r2;
        acc[k].y = acc[k].y * r1 + ao.y * r2;
        acc[k].z = acc[k].z * r1 + ao.z * r2;
        acc[k].w = acc[k].w * r1 + ao.w * r2;
      }
      L = L * r1 + Lo * r2;
      M = Mn;
    }
    if (grp != 0) return;
  }
  if (n >= G) return;
#pragma unroll
  for (int k = 0; k < kCols; ++k) write_row(n, c + k * kLanes, acc[k], L);
}

// Split merge, one item per call, one warp. Partials are read through L2 (ld.global.cg): other
// SMs wrote them. Pieces are folded in with a running maximum; each piece's max, sum and row
// (chunk) arrive in the same round trip, issued before any of them is used (ordered volatile
// loads), and the loops stop at the lane's last piece so a short merge executes only the
// instructions of its pieces.
//   * q == 1: merge_small.
//   * q > 1 (more than kMergeBatch pieces): the item is (head item / q, dimension chunk
//     item % q); lane = (piece group g, float4 column c) with 32 / q columns per chunk, group g
//     takes pieces g, g + q, ..., and the q groups are combined by xor shuffles.
template <typename T>
__device__ __forceinline__ void merge_item(const AttnParams& p, const int4& e, int item, int lane) {
  const int G = p.G;
  const int shape = e.z >> 16, q = shape & 0xff, hg = shape >> 8, ns = e.z & 0xffff;
  const float4* po4 = reinterpret_cast<const float4*>(p.ws.part_o);
  const int b = e.x / p.Hkv, h = e.x % p.Hkv;
  T* out_pair = static_cast<T*>(p.out) + static_cast<int64_t>(b) * p.out_stride + static_cast<int64_t>(h) * G * kHeadDim;
  auto write_row = [&](int n, int col, const float4& acc, float L) {
    const float inv = L > 0.f ? 1.f / L : 0.f;
    T* dst = out_pair + n * kHeadDim + col * 4;
    if (aligned(dst, 8)) {
      *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<T>(acc.x * inv, acc.y * inv), pack2<T>(acc.z * inv, acc.w * inv));
    } else {
      dst[0] = from_float<T>(acc.x * inv);
      dst[1] = from_float<T>(acc.y * inv);
      dst[2] = from_float<T>(acc.z * inv);
      dst[3] = from_float<T>(acc.w * inv);
    }
  };
  auto fold = [](float& M, float& L, float4& acc, const float2& ml, const float4& v) {
    if (ml.x != -INFINITY) {
      const float Mn = fmaxf(M, ml.x);
      const float r = M != -INFINITY ? ex2(M - Mn) : 0.f;
      const float w = ex2(ml.x - Mn);
      acc.x = acc.x * r + w * v.x;
      acc.y = acc.y * r + w * v.y;
      acc.z = acc.z * r + w * v.z;
      acc.w = acc.w * r + w * v.w;
      L = L * r + w * ml.y;
      M = Mn;
    }
  };

  if (q == 1) {
    merge_small<T>(p, e, item, lane, hg == 1, write_row);
    return;
  }

  const int n = item / q, chunk = item % q;
  const int lq = __ffs(q) - 1;       // q is a power of two
  const int lc = 5 - lq;             // log2 of the float4 columns per chunk
  const int c = lane & ((1 << lc) - 1), g = lane >> lc;
  const int col = (chunk << lc) + c;  // float4 column of the 128-dim row
  float M = -INFINITY, L = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = g; s0 < ns; s0 += q * kMergeBatch) {
    float2 ml[kMergeBatch];
    float4 v[kMergeBatch];
    const int cnt = min(kMergeBatch, (ns - s0 + q - 1) >> lq);
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) {
      if (i >= cnt) break;
      const int64_t row = static_cast<int64_t>(e.y + s0 + (i << lq)) * G + n;
      ml[i] = ld_cg_f2(&p.ws.part_ml[row]);
      v[i] = ld_cg_f4(po4 + row * (kHeadDim / 4) + col);
    }
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) {
      if (i >= cnt) break;
      after_loads(ml[i], v[i]);
    }
#pragma unroll
    for (int i = 0; i < kMergeBatch; ++i) {
      if (i >= cnt) break;
      fold(M, L, acc, ml[i], v[i]);
    }
  }
  for (int off = 1 << lc; off < 32; off <<= 1) {
    const float Mo = __shfl_xor_sync(0xffffffffu, M, off);
    const float Lo = __shfl_xor_sync(0xffffffffu, L, off);
    float4 ao;
    ao.x = __shfl_xor_sync(0xffffffffu, acc.x, off);
    ao.y = __shfl_xor_sync(0xffffffffu, acc.y, off);
    ao.z = __shfl_xor_sync(0xffffffffu, acc.z, off);
    ao.w = __shfl_xor_sync(0xffffffffu, acc.w, off);
    const float Mn = fmaxf(M, Mo);
    const float r1 = M != -INFINITY ? ex2(M - Mn) : 0.f;
    const float r2 = Mo != -INFINITY ? ex2(Mo - Mn) : 0.f;
    acc.x = acc.x * r1 + ao.x * r2;
    acc.y = acc.y * r1 + ao.y * r2;
    acc.z = acc.z * r1 + ao.z * r2;
    acc.w = acc.w * r1 + ao.w * r2;
    L = L * r1 + Lo * r2;
    M = Mn;
  }
  if (g == 0) write_row(n, col, acc, L);
}

// A split-pair entry is used only if it fits this call's shape (see unit_items).
__device__ __forceinline__ bool entry_ok(const int4& e, const AttnParams& p) {
  const int shape = e.z >> 16, q = shape & 0xff, hg = shape >> 8, ns = e.z & 0xffff;
  const int w0 = e.w & 0xffff, n_w = e.w >> 16;
  const bool shape_ok = (q == 1 && hg == 4 && ns <= 4) || (q == 1 && hg == 1 && ns > 4 && ns <= kMergeBatch) ||
                        (hg == 1 && (q == 2 || q == 4 || q == 8 || q == 16 || q == 32));
  return e.x >= 0 && e.x < p.num_pairs && e.y >= 0 && e.y + ns <= p.max_slots && shape_ok &&
         w0 + n_w <= static_cast<int>(gridDim.x) * kWarps && (ns == 0) == (n_w == 0);
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag == v (a worker warp's publication stamp), for at most kWaitLimitNs.
__device__ __forceinline__ bool flag_wait(const int* flag, int v) {
  if (ld_acquire_gpu(flag) == v) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_gpu(flag) != v) {
    __nanosleep(32);  // each poll waits for its load; the sleep only spaces the polls a little
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

template <int NT>
struct AttnSmem {
  static constexpr int kQSlot = 8 * NT * kHeadDim * 2;           // query rows of one unit
  static constexpr int kPerWarp = kStages * kStageBytes + kQSlot;  // multiple of 1024
  static constexpr int kOffBars = kWarps * kPerWarp;
  static constexpr int kBarsPerWarp = kStages + 2;  // stages, query slot, one scratch word
  static constexpr int kTotal = kOffBars + kWarps * kBarsPerWarp * 8;
  static constexpr size_t kDynamic = size_t(kTotal) + 1024;  // + alignment slack
  static_assert(kPerWarp % 1024 == 0, "per-warp regions must keep 1024-byte alignment");
};

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
  uint32_t* qdep_slot = reinterpret_cast<uint32_t*>(full + kStages + 1);  // see the query-slot reuse below

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

  // This worker's unit range and its first unit record, in one round trip. The plan is read
  // before waiting for the preceding kernel when the host knows that kernel did not write it
  // (the plan was followed by an earlier attention launch on this workspace).
  const int gw = static_cast<int>(blockIdx.x) * kWarps + warp;
  // Plan data is read once per layer launch: it is kept in L2 with an evict-last hint (the K/V
  // stream is loaded evict-first).
  const uint64_t keep = l2_policy_evict_last();
  int4 r0 = make_int4(0, 0, 0, 0);
  auto load_plan = [&]() {
    if (lane < 3)
      r0 = ld_hint(&p.ws.warp_rec[3 * gw + lane], keep);
    else if (lane == 3)
      r0.x = ld_hint(&p.ws.warp_rec[3 * (gw + 1)].x, keep);
    else if (lane == 4)
      r0.x = ld_hint(&p.ws.header[kHdrWarps], keep);
    else if (lane == 5)
      r0.x = ld_hint(&p.ws.header[kHdrUnits], keep);
    else if (lane == 6)
      r0.x = ld_hint(&p.ws.header[kHdrSplitPairs], keep);
    else if (lane == 7)
      r0 = ld_hint(&p.ws.merge_rec[gw], keep);
  };
  if (p.plan_ready) load_plan();
  // With the plan complete and the cache and tables untouched by the preceding kernel, the
  // first kStages K/V tiles are requested before waiting for that kernel (below); otherwise
  // everything below reads data produced by earlier work on the stream.
  const bool early = p.plan_ready && p.prefetch_kv;
  if (!early) {
    pdl_wait_primary();
    pdl_launch_dependents();
    if (!p.plan_ready) load_plan();
  }

  const int G = p.G;
  const int Hkv = p.Hkv;
  const int total_warps = static_cast<int>(gridDim.x) * kWarps;
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

  const int u_beg = __shfl_sync(0xffffffffu, r0.x, 0);
  const int u_end = __shfl_sync(0xffffffffu, r0.x, 3);
  const int planned_warps = __shfl_sync(0xffffffffu, r0.x, 4);
  const int planned_units = __shfl_sync(0xffffffffu, r0.x, 5);
  const int n_entries = min(max(__shfl_sync(0xffffffffu, r0.x, 6), 0), p.num_pairs);
  const int4 mr = shfl4(r0, 7);  // this warp's share of the split merge
  int n_units = u_end - u_beg;
  if (!(planned_warps == total_warps && planned_units <= p.max_units && u_beg >= 0 && u_beg <= u_end &&
        u_end <= planned_units)) {
    if (lane == 0 && n_units != 0) atomicOr(&g_deverr_attn, AEG_DEVERR_PLAN_MISMATCH);
    n_units = 0;
  }

  // Unit records, one per lane: lane (k % 32) holds the record of the worker's unit k for the
  // 32 units from the one being computed on; each finished unit's lane loads the unit 32 ahead.
  // Unit 0 is also kept in fa/fb, so that starting it does not wait for the other lanes' loads.
  const int4 fa = shfl4(r0, 1), fb = shfl4(r0, 2);
  int4 ra = fa, rb = fb;
  if (lane > 0) {
    if (lane < n_units) {
      ra = ld_hint(&p.ws.units[2 * (u_beg + lane)], keep);
      rb = ld_hint(&p.ws.units[2 * (u_beg + lane) + 1], keep);
    } else {
      ra = make_int4(0, 0, 0, -1);
      rb = make_int4(0, 0, 0, 0);
    }
  }

  // Query rows of unit k into the query slot (completes on qbar). A unit whose record is not
  // usable still completes the phase, so that the consumer's phases stay in step.
  auto rec = [&](int k, int4& a, int4& bb) {
    if (k == 0) {
      a = fa;
      bb = fb;
    } else {
      a = shfl4(ra, k & 31);
      bb = shfl4(rb, k & 31);
    }
  };
  // The slot's previous rows were read into registers with plain shared loads before this is
  // called (the caller consumes them first), so the bulk copy cannot overtake those reads.
  auto load_q = [&](int k) {
    int4 a, bb;
    rec(k, a, bb);
    if (unit_items(a, bb, p) == 0) {
      if (lane == 0) mbar_arrive(qbar);
      return;
    }
    const int b = a.x / Hkv, h = a.x % Hkv;
    const T* qsrc = q + static_cast<int64_t>(b) * p.q_stride + static_cast<int64_t>(h) * G * kHeadDim;
    const uint32_t qbytes = G * kHeadDim * 2;
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
  };

  // Issue walker: requests the tiles of the worker's units in order, kStages ahead of the
  // consumer. Items 0..2 of a unit come with its record; later ones from a 32-entry chunk of
  // the block table loaded when the walker enters the unit.
  int ik = -1, ii = 0, in_ = 0, ih = 0, ibf0 = 0, ibf1 = 0, ibf2 = 0, itbase = 0, itbl = 0;
  const int* itab = p.tables;
  int sblk[kStages];      // block id of the tile in each stage (fused cache write)
  bool patched[kStages];  // the stage holds generic-proxy writes (fused cache write patch)
#pragma unroll
  for (int i = 0; i < kStages; ++i) {
    sblk[i] = 0;
    patched[i] = false;
  }
  auto issue_enter = [&](int k) {
    ik = k;
    ii = 0;
    in_ = 0;
    if (k >= n_units) return;
    int4 a, bb;
    rec(k, a, bb);
    in_ = unit_items(a, bb, p);
    if (in_ == 0) return;
    ih = a.x % Hkv;
    ibf0 = bb.y;
    ibf1 = bb.z;
    ibf2 = bb.w;
    itab = p.tables + static_cast<int64_t>(a.x / Hkv) * p.table_stride + a.y;
    itbase = 3;
    itbl = (in_ > 3 && lane < min(32, in_ - 3)) ? itab[3 + lane] : 0;
  };
  auto issue_one = [&]() -> bool {
    while (ik < n_units && ii >= in_) issue_enter(ik + 1);
    if (ik >= n_units) return false;
    int blk;
    if (ii < 3) {
      blk = ii == 0 ? ibf0 : (ii == 1 ? ibf1 : ibf2);
    } else {
      if (ii - itbase >= 32) {
        itbase = ii;
        itbl = lane < min(32, in_ - ii) ? itab[ii + lane] : 0;
      }
      blk = __shfl_sync(0xffffffffu, itbl, ii - itbase);
    }
    const uint32_t st = g_iss % kStages;
    bool fence = false;
#pragma unroll
    for (int i = 0; i < kStages; ++i)
      if (i == static_cast<int>(st)) {
        sblk[i] = blk;
        fence = patched[i];
        patched[i] = false;
      }
    // A stage the warp only read needs no proxy fence before the TMA refill (the reads have
    // completed: their results fed the MMAs); one the fused cache write patched with generic
    // stores does.
    if (fence) fence_proxy_async_smem();
    if (lane == 0) {
      if (static_cast<unsigned long long>(static_cast<long long>(blk)) >= static_cast<unsigned long long>(p.num_blocks))
        atomicOr(&g_deverr_attn, AEG_DEVERR_BLOCK_ID_RANGE);  // TMA zero-fills it
      if (!abort) {
        uint8_t* dst = ring + st * kStageBytes;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        tma_load_5d(dst, &kmap, &full[st], 0, 0, 0, ih, blk, pol);
        tma_load_5d(dst + kBoxBytes, &vmap, &full[st], 0, 0, 0, ih, blk, pol);
      }
    }
    ++g_iss;
    ++ii;
    return true;
  };
  auto refill = [&]() {
    while (g_iss - g_con < kStages && issue_one()) {
    }
  };

  if (early) {
    refill();
    // The first unit's query rows are requested into L2 only (no data reaches the SM before the
    // wait), so that their load after the wait is an L2 hit.
    // Every address lies inside the rows: the row start, then the starts of the later lines.
    if (n_units > 0 && unit_items(fa, fb, p) > 0) {
      const T* qrow = q + static_cast<int64_t>(fa.x / Hkv) * p.q_stride +
                      static_cast<int64_t>(fa.x % Hkv) * G * kHeadDim;
      const uintptr_t a0 = reinterpret_cast<uintptr_t>(qrow);
      const uintptr_t line0 = a0 & ~static_cast<uintptr_t>(127);
      const uintptr_t a1 = a0 + static_cast<uintptr_t>(G) * kHeadDim * sizeof(T);
      if (lane < static_cast<int>((a1 - line0 + 127) / 128))
        prefetch_l2(reinterpret_cast<const void*>(lane == 0 ? a0 : line0 + 128 * static_cast<uintptr_t>(lane)));
    }
    pdl_wait_primary();
    pdl_launch_dependents();
  }
  if (n_units > 0) load_q(0);
  refill();
  // Launches with this plan so far: this warp's own flag, which every worker warp of every
  // earlier launch stamped once. The previous launch wrote it and has finished (the wait above),
  // so a relaxed load sees it; issued after the first tiles, it delays nothing, and its value
  // is needed only when this warp publishes.
  const int epoch_word = lane == 0 ? ld_relaxed_gpu(&p.ws.warp_flag[gw * kFlagStride]) : 0;

  for (int c = 0; c < n_units; ++c) {
    if (c > 0 && lane == ((c - 1) & 31) && c + 31 < n_units) {
      ra = p.ws.units[2 * (u_beg + c + 31)];
      rb = p.ws.units[2 * (u_beg + c + 31) + 1];
    }
    int4 ua, ub;
    rec(c, ua, ub);
    const int n = unit_items(ua, ub, p);
    if (n == 0 && lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_PLAN_MISMATCH);
    const int b = ua.x / Hkv, h = ua.x % Hkv, j0 = ua.y, slot = ua.w, n_ctx = ub.x;

    // Query fragments (B operand of S^T = K Q^T) from the query slot; then the slot is free for
    // the next unit's rows.
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
    // The next unit's rows overwrite the slot: make every lane's slot reads complete first (a
    // store of a value computed from all of them cannot issue before they have returned).
    {
      uint32_t dep = 0;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) dep ^= qf[nt][ks][0] ^ qf[nt][ks][1];
      if (lane == 0) *qdep_slot = dep;
    }
    __syncwarp();
    if (c + 1 < n_units) load_q(c + 1);
    if (n == 0) continue;

    // Fused cache write (or the refresh of a row written just before): this unit reads the block
    // of position n_ctx - 1.
    const bool last = (p.fuse_write || p.refresh_last) && n_ctx > 0 &&
                      j0 + n == (n_ctx + kBlockTokens - 1) / kBlockTokens;
    uint2 knew = make_uint2(0u, 0u), vnew = make_uint2(0u, 0u);
    if (last && !p.fuse_write) {
      // The newest row of head h as the preceding kernel left it (read after the wait, through
      // L2); the block id comes from the unit record when it holds it, else from the table.
      const int il = n - 1;
      const int blk = il == 0 ? ub.y : il == 1 ? ub.z : il == 2 ? ub.w
                    : p.tables[static_cast<int64_t>(b) * p.table_stride + (n_ctx - 1) / kBlockTokens];
      if (static_cast<unsigned long long>(static_cast<long long>(blk)) < static_cast<unsigned long long>(p.num_blocks)) {
        const int64_t off = static_cast<int64_t>(blk) * p.block_stride +
                            (static_cast<int64_t>((n_ctx - 1) % kBlockTokens) * Hkv + h) * kHeadDim + 4 * lane;
        knew = __ldcg(reinterpret_cast<const uint2*>(static_cast<const T*>(p.k_cache) + off));
        vnew = __ldcg(reinterpret_cast<const uint2*>(static_cast<const T*>(p.v_cache) + off));
      }
    } else if (last) {
      const uint32_t* kn = reinterpret_cast<const uint32_t*>(static_cast<const T*>(p.k_new) +
                                                             static_cast<int64_t>(b) * p.k_new_stride +
                                                             static_cast<int64_t>(h) * kHeadDim) + 2 * lane;
      const uint32_t* vn = reinterpret_cast<const uint32_t*>(static_cast<const T*>(p.v_new) +
                                                             static_cast<int64_t>(b) * p.v_new_stride +
                                                             static_cast<int64_t>(h) * kHeadDim) + 2 * lane;
      knew = make_uint2(kn[0], kn[1]);
      vnew = make_uint2(vn[0], vn[1]);
    }

    float o[8][NT][4];
    float m[NT][2], l[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
    }

    for (int k = 0; k < n; ++k) {
      const uint32_t st = g_con % kStages, ph = (g_con / kStages) & 1;
      if (!abort && !mbar_wait_bounded(&full[st], ph, kWaitLimitNs)) report_timeout();
      const int j = j0 + k;
      const int nvalid = min(kBlockTokens, n_ctx - j * kBlockTokens);
      if (!abort && nvalid > 0) {
        const uint32_t kbase = smem_u32(ring + st * kStageBytes);
        const uint32_t vbase = kbase + kBoxBytes;
        if (last && k == n - 1) {
          // Fused cache write: store the newest token's K/V row of head h in the cache (no other
          // reader of that row in this launch: other warps read other heads' rows) and patch it
          // into the swizzled tiles, which were fetched before the store.
          int blk = 0;
#pragma unroll
          for (int i = 0; i < kStages; ++i)
            if (i == static_cast<int>(st)) blk = sblk[i];
          const int t = (n_ctx - 1) % kBlockTokens;
          if (p.fuse_write && static_cast<unsigned long long>(static_cast<long long>(blk)) <
                                  static_cast<unsigned long long>(p.num_blocks)) {
            const int64_t off = static_cast<int64_t>(blk) * p.block_stride +
                                (static_cast<int64_t>(t) * Hkv + h) * kHeadDim + 4 * lane;
            *reinterpret_cast<uint2*>(static_cast<T*>(p.k_cache) + off) = knew;
            *reinterpret_cast<uint2*>(static_cast<T*>(p.v_cache) + off) = vnew;
          }
          const int half = lane >> 4, ch = (lane & 15) >> 1;
          const uint32_t soff = (half * kBlockTokens + t) * 128 + ((ch ^ (t & 7)) << 4) + (lane & 1) * 8;
          *reinterpret_cast<uint2*>(ring + st * kStageBytes + soff) = knew;
          *reinterpret_cast<uint2*>(ring + st * kStageBytes + kBoxBytes + soff) = vnew;
          __syncwarp();
#pragma unroll
          for (int i = 0; i < kStages; ++i)
            if (i == static_cast<int>(st)) patched[i] = true;
        }

        // S^T[16 tokens][8 heads] per n-tile.
        float s[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int tok = lr + ((lm & 1) << 3);
          const int cc = ks * 2 + (lm >> 1);
          const uint32_t addr = kbase + ((cc >> 3) * kBlockTokens + tok) * 128 + (((cc & 7) ^ lr) << 4);
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
          const int cc = mt * 2 + (lm & 1);
          const uint32_t addr = vbase + ((cc >> 3) * kBlockTokens + tok) * 128 + (((cc & 7) ^ lr) << 4);
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
      refill();
    }

    // ---- unit result ----
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        l[nt][0] += __shfl_xor_sync(0xffffffffu, l[nt][0], off);
        l[nt][1] += __shfl_xor_sync(0xffffffffu, l[nt][1], off);
      }
    if (slot < 0) {
      T* ob = out + static_cast<int64_t>(b) * p.out_stride + static_cast<int64_t>(h) * G * kHeadDim;
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
      const int64_t base = static_cast<int64_t>(slot) * G;
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
  }

  // The first split-pair entry of this warp's merge share (plan data, read early).
  int entry = mr.x, k = mr.y;
  const bool share_ok = planned_warps == total_warps && mr.z >= 0 && entry >= 0 && entry <= n_entries;
  const int4 none = make_int4(-1, 0, (1 | (1 << 8)) << 16, 0);
  int4 me = (share_ok && mr.z > 0 && entry < n_entries) ? p.ws.split_pairs[entry] : none;

  const int epoch = __shfl_sync(0xffffffffu, epoch_word, 0);
  const int stamp = static_cast<int>(static_cast<unsigned>(epoch) + 1u);  // this launch's flag value

  // Publish this warp's partials: the lanes meet, then lane 0 stamps the warp's flag with a
  // release store. The warp barrier orders every lane's partial stores before that store, and a
  // release is cumulative, so a reader that acquires the stamp sees all of them. Warps publish
  // independently: a merge waits only for the warps that computed its pair's pieces.
  __syncwarp();
  if (lane == 0) st_release_gpu(&p.ws.warp_flag[gw * kFlagStride], stamp);

  // The split merge: the plan spreads the merge items evenly over all warps; an item waits
  // only for the flags of the warps that computed its pair's pieces (lanes watch up to 32 of
  // them at once). Warps publish before they merge and all CTAs of the grid are resident
  // together (one per SM), so the waits end; they are bounded all the same.
  int ready_entry = -1;  // entry whose producer CTAs are known to have published
  if (share_ok) {
    for (int left = mr.z; left > 0; --left) {
      if (k >= merge_items(me.z >> 16, G)) {  // next split-pair entry
        ++entry;
        k = 0;
        me = entry < n_entries ? p.ws.split_pairs[entry] : none;
      }
      if (!entry_ok(me, p) || k < 0) {
        if (lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_PLAN_MISMATCH);
        break;
      }
      if (ready_entry != entry) {
        const int w0 = me.w & 0xffff, nw = me.w >> 16;
        int ok = 1;
        for (int i = 0; i < nw && ok; i += 32) {
          const int ww = w0 + i + lane;
          ok = __all_sync(0xffffffffu,
                          i + lane >= nw || ww == gw || flag_wait(&p.ws.warp_flag[ww * kFlagStride], stamp));
        }
        __syncwarp();  // orders the lanes' acquiring flag reads before every lane's partial loads
        if (!ok) {
          if (lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_WAIT_TIMEOUT);
          break;
        }
        ready_entry = entry;
      }
      merge_item<T>(p, me, k, lane);
      ++k;
    }
  } else if (lane == 0) {
    atomicOr(&g_deverr_attn, AEG_DEVERR_PLAN_MISMATCH);
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

// Checks that the attention kernel can be configured on the current device and that its grid
// fits the workspace's worker-warp capacity; enqueues nothing.
template <typename T, int NT>
int check_attn_t(int max_warps) {
  const int per_sm = attn_ctas_per_sm<T, NT>();
  if (per_sm < 1) {
    (void)cudaGetLastError();
    return set_error(AEG_ERR_CUDA, "decode attention kernel cannot be configured on this device");
  }
  if (num_sms() * per_sm * kWarps > max_warps)
    return set_error(AEG_ERR_UNSUPPORTED, "decode: %d worker warps exceed the workspace's %d", num_sms() * per_sm * kWarps,
                     max_warps);
  return AEG_OK;
}

// `started` (may be null): an event that fires once every CTA of this launch has started
// (programmatic event triggered at block start); see LaunchOrder.
template <typename T, int NT>
int launch_attn_t(const CUtensorMap& km, const CUtensorMap& vm, const AttnParams& prm, cudaStream_t stream,
                  cudaEvent_t started) {
  const int per_sm = attn_ctas_per_sm<T, NT>();
  // One CTA per SM (the occupancy limit), so all CTAs of the grid are resident together once the
  // preceding kernels have left the SMs; the split merge's waits on other CTAs rely on that.
  // Not a cooperative launch: a cooperative grid does not start early under programmatic
  // dependent launch (measured: cfg2 step 0.506 -> 0.439 ms without it). The next layer's grid
  // cannot take SMs before every CTA of this one has started (it launches only when all of them
  // have passed griddepcontrol.launch_dependents), and every wait is bounded.
  cudaLaunchAttribute attr[2] = {pdl_attr(), cudaLaunchAttribute{}};
  unsigned n_attr = 1;
  if (started != nullptr) {
    attr[1].id = cudaLaunchAttributeProgrammaticEvent;
    attr[1].val.programmaticEvent.event = started;
    attr[1].val.programmaticEvent.flags = 0;
    attr[1].val.programmaticEvent.triggerAtBlockStart = 1;
    n_attr = 2;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms() * per_sm));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = AttnSmem<NT>::kDynamic;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = n_attr;
  AEG_CHECK_CUDA(cudaLaunchKernelEx(&cfg, decode_attn_kernel<T, NT>, km, vm, prm));
  return AEG_OK;
}

// Worker warps of an attention launch on the current device (the plan cuts the work into this
// many ranges; the attention kernel checks that its grid matches).
int worker_warps(int G) {
  const int per_sm = ctas_per_sm(AEG_DTYPE_FP16, G <= 8 ? 1 : 2);
  return num_sms() * (per_sm > 0 ? per_sm : 1) * kWarps;
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

// Workspaces whose plan was launched and not yet followed by an attention launch: the first
// attention launch after a plan may directly follow the plan kernel, so it reads the plan only
// after waiting for the preceding kernel; later launches read it before.
std::mutex g_fresh_mu;
std::unordered_set<const void*> g_fresh_plans;

void mark_plan_fresh(const void* ws) {
  std::lock_guard<std::mutex> lock(g_fresh_mu);
  g_fresh_plans.insert(ws);
}

bool take_plan_fresh(const void* ws) {
  std::lock_guard<std::mutex> lock(g_fresh_mu);
  return g_fresh_plans.erase(ws) > 0;
}

// Everything an attention launch needs, checked and built on the host before anything is
// enqueued: the K/V tensor maps and the kernel parameters (plan_ready is set by the caller).
struct DecodeLaunch {
  CUtensorMap km, vm;
  AttnParams prm;
  int dtype;
  int nt;
};

int decode_prepare(DecodeLaunch* dl, void* out, int64_t out_stride, const void* q, int64_t q_stride,
                   const void* k_new, int64_t k_new_stride, const void* v_new, int64_t v_new_stride, void* k_cache,
                   void* v_cache, int64_t block_stride, int64_t num_blocks, const int32_t* block_tables,
                   int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale, int dtype,
                   void* workspace, size_t workspace_bytes, bool fuse, int flags, const WsLayout& L) {
  AEG_CHECK_ARG(dtype == AEG_DTYPE_FP16 || dtype == AEG_DTYPE_BF16, "decode: dtype %d is not fp16/bf16", dtype);
  AEG_CHECK_ARG(out && q && k_cache && v_cache && block_tables && seq_lens, "decode: null pointer");
  AEG_CHECK_ARG(workspace != nullptr && aligned(workspace, 256), "decode: workspace must be 256-byte aligned");
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
  const int nt = Hq / Hkv <= 8 ? 1 : 2;
  int st = dtype == AEG_DTYPE_BF16 ? (nt == 1 ? check_attn_t<__nv_bfloat16, 1>(L.max_warps)
                                               : check_attn_t<__nv_bfloat16, 2>(L.max_warps))
                                   : (nt == 1 ? check_attn_t<__half, 1>(L.max_warps) : check_attn_t<__half, 2>(L.max_warps));
  if (st != AEG_OK) return st;
  st = encode_kv_map(&dl->km, k_cache, dtype, Hkv, block_stride, num_blocks);
  if (st != AEG_OK) return st;
  st = encode_kv_map(&dl->vm, v_cache, dtype, Hkv, block_stride, num_blocks);
  if (st != AEG_OK) return st;

  AttnParams& prm = dl->prm;
  prm = AttnParams{};
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
  prm.max_warps = L.max_warps;
  prm.max_units = L.max_units;
  prm.max_slots = L.max_slots;
  prm.num_blocks = num_blocks;
  prm.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);  // log2(e)
  prm.q_bulk = (aligned(q, 16) && q_stride % 8 == 0) ? 1 : 0;
  prm.plan_ready = 0;
  prm.prefetch_kv = (flags & (AEG_DECODE_PREFETCH | AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE)) ? 1 : 0;
  prm.fuse_write = fuse ? 1 : 0;
  prm.refresh_last = (!fuse && (flags & AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE) && !(flags & AEG_DECODE_PREFETCH)) ? 1 : 0;
  prm.k_new = k_new;
  prm.v_new = v_new;
  prm.k_new_stride = k_new_stride;
  prm.v_new_stride = v_new_stride;
  prm.k_cache = k_cache;
  prm.v_cache = v_cache;
  prm.block_stride = block_stride;
  prm.ws = ws_ptrs(workspace, L);
  dl->dtype = dtype;
  dl->nt = nt;
  return AEG_OK;
}

// Order of attention launches on one device across streams.
//
// The split merge waits for other CTAs of its own grid, which is safe only if the whole grid is
// resident together. On one stream that holds: a launch starts only when every CTA of the
// previous one has started (programmatic dependent launch) or that kernel has finished. Two
// grids on two streams could each hold part of the SMs and wait for CTAs that cannot start
// until the other grid leaves; the bounded waits would then time out. So every eager launch
// carries a programmatic event that fires once all of its CTAs have started, and a launch on a
// different stream than the device's previous attention launch first waits for that event (as
// a programmatic dependency: its CTAs may start early but proceed past griddepcontrol.wait only
// when that grid has finished). Each grid therefore starts only after the previous one is fully
// resident, so at most one grid is ever partially resident and every wait ends. Launches made
// while a stream is being captured into a CUDA graph are not ordered this way: graphs that
// hold attention launches must be replayed on one stream or on streams the caller orders.
class LaunchOrder {
 public:
  ~LaunchOrder() { if (locked_) mu_of(dev_).unlock(); }

  // Locks the device's order and, if needed, makes `s` wait for the previous launch's start.
  // On return event() is the event to attach to the launch (null when not ordering).
  int enter(cudaStream_t s, bool* waited) {
    *waited = false;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    AEG_CHECK_CUDA(cudaStreamIsCapturing(s, &cs));
    if (cs != cudaStreamCaptureStatusNone) return AEG_OK;
    AEG_CHECK_CUDA(cudaGetDevice(&dev_));
    if (dev_ < 0 || dev_ >= kDevices)
      return set_error(AEG_ERR_UNSUPPORTED, "decode: device ordinal %d >= %d", dev_, kDevices);
    mu_of(dev_).lock();
    locked_ = true;
    State& st = state()[dev_];
    if (st.started == nullptr) AEG_CHECK_CUDA(cudaEventCreateWithFlags(&st.started, cudaEventDisableTiming));
    if (st.any && st.last != s) {
      AEG_CHECK_CUDA(cudaStreamWaitEvent(s, st.started, 0));
      *waited = true;
    }
    stream_ = s;
    return AEG_OK;
  }
  cudaEvent_t event() const { return locked_ ? state()[dev_].started : nullptr; }
  // Records that the launch carrying event() was made on the stream given to enter().
  void launched() {
    if (!locked_) return;
    State& st = state()[dev_];
    st.last = stream_;
    st.any = true;
  }

 private:
  static constexpr int kDevices = 64;
  struct State {
    cudaEvent_t started = nullptr;
    cudaStream_t last = nullptr;
    bool any = false;
  };
  static State* state() {
    static State s[kDevices];
    return s;
  }
  static std::mutex& mu_of(int dev) {
    static std::mutex m[kDevices];
    return m[dev];
  }
  int dev_ = -1;
  bool locked_ = false;
  cudaStream_t stream_ = nullptr;
};

int decode_launch(const DecodeLaunch& dl, cudaStream_t s, LaunchOrder& order) {
  cudaEvent_t ev = order.event();
  int st;
  if (dl.dtype == AEG_DTYPE_BF16)
    st = dl.nt == 1 ? launch_attn_t<__nv_bfloat16, 1>(dl.km, dl.vm, dl.prm, s, ev)
                    : launch_attn_t<__nv_bfloat16, 2>(dl.km, dl.vm, dl.prm, s, ev);
  else
    st = dl.nt == 1 ? launch_attn_t<__half, 1>(dl.km, dl.vm, dl.prm, s, ev) : launch_attn_t<__half, 2>(dl.km, dl.vm, dl.prm, s, ev);
  if (st == AEG_OK) order.launched();
  return st;
}

int decode_common(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_new,
                  int64_t k_new_stride, const void* v_new, int64_t v_new_stride, void* k_cache, void* v_cache,
                  int64_t block_stride, int64_t num_blocks, const int32_t* block_tables, int table_stride,
                  const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale, int dtype, void* workspace,
                  size_t workspace_bytes, void* stream, bool fuse, int flags) {
  int st = validate_shape(B, Hq, Hkv, D, table_stride);
  if (st != AEG_OK) return st;
  if (B == 0) return AEG_OK;
  DecodeLaunch dl;
  st = decode_prepare(&dl, out, out_stride, q, q_stride, k_new, k_new_stride, v_new, v_new_stride, k_cache, v_cache,
                      block_stride, num_blocks, block_tables, table_stride, seq_lens, B, Hq, Hkv, D, scale, dtype,
                      workspace, workspace_bytes, fuse, flags, ws_layout(B, Hq, Hkv, D));
  if (st != AEG_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchOrder order;
  bool waited = false;
  st = order.enter(s, &waited);
  if (st != AEG_OK) return st;
  dl.prm.plan_ready = take_plan_fresh(workspace) ? 0 : 1;
  // After a wait for another stream's grid, that grid is a programmatic predecessor of this
  // launch too: request no tiles before the grid-dependency wait.
  if (waited) dl.prm.prefetch_kv = 0;
  return decode_launch(dl, s, order);
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
//     layout sized for this device's worker warps W (1184 on a 148-SM B200) instead of the
//     largest supported count: partial rows for 2 * W units and unit records for B*Hkv + W, so
//     the need grows with the GQA group and B*Hkv: about 8.5 MB for 64 sequences x 4 KV heads
//     x 7 query heads each. A call that would need more is rejected with
//     AEG_ERR_INVALID_ARGUMENT before anything is enqueued.
//   * Nothing in the scratch has to start at zero for the first call: the plan kernel that
//     every call enqueues rewrites the header, the warp, unit, split-pair and merge records,
//     and sets every worker warp's publication flag to zero. The attention kernel then stamps
//     each worker warp's flag with (its value at launch) + 1 once that warp's partials are
//     stored, and a merge item waits for that stamp from each warp that computed a piece of its
//     pair; the partial rows are written before they are read. (Static device memory also
//     starts zeroed when the module is loaded.)
//   * A call that fails a check (arguments, sizes, alignment, tensor-map encoding) returns its
//     error before enqueuing anything, so it leaves the scratch as the previous call left it.
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
  const int W = aeg::worker_warps(Hq / Hkv);
  if (W > L.max_warps)
    return aeg::set_error(AEG_ERR_UNSUPPORTED, "decode_plan: %d worker warps exceed the workspace's %d", W, L.max_warps);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  aeg::WsPtrs w = aeg::ws_ptrs(workspace, L);
  aeg::decode_plan_kernel<<<1, aeg::kPlanThreads, 0, s>>>(seq_lens, block_tables, B, Hkv, Hq / Hkv, table_stride, W, w);
  AEG_CHECK_LAUNCH("decode_plan");
  aeg::mark_plan_fresh(workspace);
  return AEG_OK;
}

int aeg_paged_attn_decode(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_cache,
                          const void* v_cache, int64_t block_stride, int64_t num_blocks, const int32_t* block_tables,
                          int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale,
                          int dtype, void* workspace, size_t workspace_bytes, int flags, void* stream) {
  return aeg::decode_common(out, out_stride, q, q_stride, nullptr, 0, nullptr, 0, const_cast<void*>(k_cache),
                            const_cast<void*>(v_cache), block_stride, num_blocks, block_tables, table_stride, seq_lens, B,
                            Hq, Hkv, D, scale, dtype, workspace, workspace_bytes, stream, false, flags);
}

int aeg_decode_layer(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* key_new,
                     int64_t key_stride, const void* value_new, int64_t value_stride, void* k_cache, void* v_cache,
                     int64_t block_stride, int64_t num_blocks, const int32_t* block_tables, int table_stride,
                     const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale, int dtype, void* workspace,
                     size_t workspace_bytes, int flags, void* stream) {
  return aeg::decode_common(out, out_stride, q, q_stride, key_new, key_stride, value_new, value_stride, k_cache, v_cache,
                            block_stride, num_blocks, block_tables, table_stride, seq_lens, B, Hq, Hkv, D, scale, dtype,
                            workspace, workspace_bytes, stream, true, flags);
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
  const int W = aeg::worker_warps(Hq / Hkv);
  const aeg::WsLayout L = aeg::layout_for(B, Hq, Hkv, D, W);
  AEG_CHECK_ARG(L.total <= aeg::kNoAllocScratchBytes,
                "decode_noalloc: B=%d, Hq=%d, Hkv=%d needs %zu bytes of scratch, more than the %zu bytes of the "
                "static scratch; use aeg_paged_attn_decode with a caller-owned workspace",
                B, Hq, Hkv, L.total, aeg::kNoAllocScratchBytes);
  void* scratch = nullptr;
  st = aeg::noalloc_scratch(&scratch);
  if (st != AEG_OK) return st;
  // Every argument check, the kernel configuration and the tensor maps come before the first
  // launch: a rejected call enqueues nothing and leaves the scratch as the last call left it.
  aeg::DecodeLaunch dl;
  st = aeg::decode_prepare(&dl, out, out_stride, q, q_stride, nullptr, 0, nullptr, 0, const_cast<void*>(k_cache),
                           const_cast<void*>(v_cache), block_stride, num_blocks, block_tables, table_stride, seq_lens, B,
                           Hq, Hkv, D, scale, dtype, scratch, aeg::kNoAllocScratchBytes, false, 0, L);
  if (st != AEG_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  aeg::LaunchOrder order;
  bool waited = false;
  st = order.enter(s, &waited);
  if (st != AEG_OK) return st;
  aeg::decode_plan_kernel<<<1, aeg::kPlanThreads, 0, s>>>(seq_lens, block_tables, B, Hkv, Hq / Hkv, table_stride, W,
                                                          aeg::ws_ptrs(scratch, L));
  AEG_CHECK_LAUNCH("decode_plan (noalloc)");
  dl.prm.plan_ready = 0;  // the plan kernel directly precedes this launch: read it after the wait
  return aeg::decode_launch(dl, s, order);
}

}  // extern "C"
