// Paged decode attention over Aegaeon's block-table KV cache, written for sm_100a.
//
// Semantics: the decode call of the vLLM 0.5.1 FlashAttention backend that the reference runs
// per layer (flash_attn_with_kvcache(q[:, None], K_l, V_l, block_table, cache_seqlens, scale,
// causal=True) reached from aegaeon/aegaeon/worker.py:517-523, metadata from worker.py:554-713).
// One query token per sequence, so every cached key j < seq_len is visible; query head h reads
// KV head h / (Hq / Hkv).
//
// Design (memory-bound: every K/V byte is read exactly once per layer call):
//   * Work unit = (sequence b, group of HG KV heads, range of 16-token blocks). A plan kernel,
//     run once per decode step, splits every (b, group) into ranges of near-equal length so
//     that all CTAs stream the same number of bytes.
//   * Persistent CTAs: HG consumer warps (one per KV head of the group) + 1 producer warp.
//     The producer streams each block's K and V boxes (16 tokens x HG heads x 128 dims) into a
//     STAGES-deep shared-memory ring with 5-D bulk-tensor TMA loads (128-byte swizzle,
//     evict-first L2 policy), completing on mbarriers. For Aegaeon's layout a (block, layer)
//     K or V box is one contiguous 16 KiB span at Hkv = 4.
//   * Consumers compute S^T = K Q^T with mma.sync m16n8k16 (16 tokens x 8 query heads of the
//     GQA group; K fragments by ldmatrix from the swizzled tile), fp32 online softmax in the
//     exp2 domain with quad shuffles, transpose P in registers with movmatrix, then
//     O^T += V^T P^T (V fragments by ldmatrix.trans). Tensor cores carry the G query heads
//     that share one K/V tile, so the CUDA cores only do the softmax.
//   * A unit that covers a whole sequence writes the output row directly. Split units write
//     fp32 partials (unnormalised O, running max, running sum); the last CTA of a (b, group)
//     to finish (atomic ticket, no spinning) merges them and resets its counter.
//   * Every mbarrier wait is bounded (2 s); a timeout raises AEG_DEVERR_WAIT_TIMEOUT and the
//     kernel drains instead of hanging.
#include "aeg_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <mutex>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_attn = 0;

constexpr int kHeadDim = 128;
constexpr int kHalves = kHeadDim / 64;   // 128-byte rows per (token, head)
constexpr int kBlockTokens = 16;
constexpr int kMaxTargetUnits = 4096;    // upper bound on the plan's balanced unit count
constexpr int kPlanThreads = 1024;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ---------------------------------------------------------------------------------------
// Workspace layout (all offsets 256-byte aligned):
//   header   : int32[64]  {num_units, chunk_blocks, num_pairs, ...}
//   counters : int32[P]   per (sequence, KV-head group) split tickets, zeroed by the plan
//   units    : int4[max_units]  {pair, j0, j1, (split << 16) | nsplit}
//   part_ml  : float2[max_units * HG * G]          (running max in log2 units, running sum)
//   part_o   : float [max_units * HG * G * D]      unnormalised partial outputs
struct WsLayout {
  size_t counters, units, part_ml, part_o, total;
  int max_units;
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

inline int pick_hg(int Hkv) { return (Hkv % 4 == 0) ? 4 : (Hkv % 2 == 0 ? 2 : 1); }

WsLayout ws_layout(int B, int Hq, int Hkv, int D) {
  WsLayout w{};
  const int hg = pick_hg(Hkv);
  const int ng = Hkv / hg;
  const int G = Hq / Hkv;
  const int64_t P = int64_t(B) * ng;
  w.max_units = static_cast<int>(kMaxTargetUnits + P);
  size_t off = 256;
  w.counters = off;
  off = align256(off + sizeof(int) * P);
  w.units = off;
  off = align256(off + sizeof(int4) * size_t(w.max_units));
  w.part_ml = off;
  off = align256(off + sizeof(float2) * size_t(w.max_units) * hg * G);
  w.part_o = off;
  off = align256(off + sizeof(float) * size_t(w.max_units) * hg * G * D);
  w.total = off;
  return w;
}

struct WsPtrs {
  int* header;
  int* counters;
  int4* units;
  float2* part_ml;
  float* part_o;
};

inline WsPtrs ws_ptrs(void* ws, const WsLayout& L) {
  char* b = static_cast<char*>(ws);
  return WsPtrs{reinterpret_cast<int*>(b), reinterpret_cast<int*>(b + L.counters), reinterpret_cast<int4*>(b + L.units),
                reinterpret_cast<float2*>(b + L.part_ml), reinterpret_cast<float*>(b + L.part_o)};
}

// ---------------------------------------------------------------------------------------
// Plan kernel (one CTA): chunk size, per-(b, group) split counts, unit list.

__device__ __forceinline__ int clamp_len(int n, int cap) {
  if (n < 0 || n > cap) {
    atomicOr(&g_deverr_attn, AEG_DEVERR_SEQ_LEN_RANGE);
    return n < 0 ? 0 : cap;
  }
  return n;
}

__global__ void __launch_bounds__(kPlanThreads)
decode_plan_kernel(const int* __restrict__ seq_lens, int B, int NG, int table_stride, int target_units,
                   WsPtrs ws) {
  __shared__ long long s_red[kPlanThreads / 32];
  __shared__ int s_scan[kPlanThreads];
  const int tid = threadIdx.x;
  const int P = B * NG;
  const int cap = table_stride * kBlockTokens;

  // Pass 1: total blocks over all (b, group) pairs.
  long long local = 0;
  for (int p = tid; p < P; p += kPlanThreads) {
    const int n = clamp_len(seq_lens[p / NG], cap);
    local += (n + kBlockTokens - 1) / kBlockTokens;
  }
  for (int o = 16; o > 0; o >>= 1) local += __shfl_xor_sync(0xffffffffu, local, o);
  if ((tid & 31) == 0) s_red[tid >> 5] = local;
  __syncthreads();
  if (tid < 32) {
    long long v = s_red[tid];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (tid == 0) s_red[0] = v;
  }
  __syncthreads();
  const long long total = s_red[0];
  const int chunk = static_cast<int>(max(1LL, (total + target_units - 1) / target_units));

  // Pass 2: each thread owns a contiguous range of pairs; exclusive scan of split counts.
  const int per = (P + kPlanThreads - 1) / kPlanThreads;
  const int p0 = min(P, tid * per), p1 = min(P, p0 + per);
  int cnt = 0;
  for (int p = p0; p < p1; ++p) {
    const int nb = (min(max(seq_lens[p / NG], 0), cap) + kBlockTokens - 1) / kBlockTokens;
    cnt += max(1, (nb + chunk - 1) / chunk);
  }
  s_scan[tid] = cnt;
  __syncthreads();
  for (int o = 1; o < kPlanThreads; o <<= 1) {
    const int v = tid >= o ? s_scan[tid - o] : 0;
    __syncthreads();
    s_scan[tid] += v;
    __syncthreads();
  }
  int u = s_scan[tid] - cnt;
  for (int p = p0; p < p1; ++p) {
    const int nb = (min(max(seq_lens[p / NG], 0), cap) + kBlockTokens - 1) / kBlockTokens;
    const int ns = max(1, (nb + chunk - 1) / chunk);
    for (int s = 0; s < ns; ++s) {
      const int j0 = static_cast<int>((static_cast<long long>(s) * nb) / ns);
      const int j1 = static_cast<int>((static_cast<long long>(s + 1) * nb) / ns);
      ws.units[u++] = make_int4(p, j0, j1, (s << 16) | ns);
    }
    ws.counters[p] = 0;
  }
  if (tid == kPlanThreads - 1) {
    ws.header[0] = s_scan[kPlanThreads - 1];
    ws.header[1] = chunk;
    ws.header[2] = P;
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
  int NG;
  int num_pairs;   // B * NG
  int max_units;   // capacity of the workspace unit list
  int64_t num_blocks;
  float scale_log2;
  WsPtrs ws;
};

// A unit read from the workspace is used only if it is consistent with this call's shape; a
// workspace that was not planned for this call (or not planned at all) is skipped and reported
// instead of steering loads out of bounds.
__device__ __forceinline__ bool unit_ok(const int4& un, int u, const AttnParams& p) {
  const int split = un.w >> 16, nsplit = un.w & 0xffff;
  return un.x >= 0 && un.x < p.num_pairs && un.y >= 0 && un.y <= un.z && un.z <= p.table_stride && nsplit >= 1 &&
         split < nsplit && u - split >= 0 && u - split + nsplit <= p.max_units;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

template <int HG>
struct Smem {
  static constexpr int kBoxBytes = HG * kHalves * kBlockTokens * 128;  // one K (or V) box
  static constexpr int kStageBytes = 2 * kBoxBytes;
};

template <int HG>
__host__ __device__ constexpr int stages_for() {
  return HG == 4 ? 3 : (HG == 2 ? 6 : 12);
}

template <int HG>
__host__ __device__ constexpr size_t attn_smem_bytes() {
  return size_t(stages_for<HG>()) * Smem<HG>::kStageBytes + 1024 /*align*/ + 1024 /*barriers + combine*/;
}

template <typename T, int HG, int NT>
__global__ void __launch_bounds__((HG + 1) * 32, 1)
decode_attn_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const AttnParams p) {
  constexpr int STAGES = stages_for<HG>();
  constexpr int kBox = Smem<HG>::kBoxBytes;
  constexpr int kHeadBytes = kHalves * kBlockTokens * 128;  // one head's 16 x 128 tile in a box
  constexpr int NCONS = HG * 32;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023) & ~1023u) - raw);
  uint8_t* tiles = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * 2 * kBox);
  uint64_t* empty = full + STAGES;
  float* s_mx = reinterpret_cast<float*>(empty + STAGES);  // [64]
  float* s_inv = s_mx + 64;                                // [64]
  volatile int* s_flag = reinterpret_cast<volatile int*>(s_inv + 64);  // [0]=last ticket, [1]=abort

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], HG);
    }
    s_flag[0] = 0;
    s_flag[1] = 0;
    fence_mbar_init();
  }
  if (warp == HG && lane == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  __syncthreads();

  // Everything below reads data produced by earlier work on the stream.
  pdl_wait_primary();
  pdl_launch_dependents();

  const int num_units = min(max(p.ws.header[0], 0), p.max_units);
  const int G = p.G;
  const int NG = p.NG;

  if (warp == HG) {
    // ------------------------------- producer warp -------------------------------------
    uint32_t stage = 0, phase = 0;
    const uint64_t pol = l2_policy_evict_first();
    bool abort = false;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const int4 un = p.ws.units[u];
      if (!unit_ok(un, u, p)) {
        if (lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_PLAN_MISMATCH);
        continue;
      }
      const int b = un.x / NG, g = un.x % NG;
      const int* tb = p.tables + static_cast<int64_t>(b) * p.table_stride;
      for (int jb = un.y; jb < un.z; jb += 32) {
        const int cnt = min(32, un.z - jb);
        const int mine = lane < cnt ? tb[jb + lane] : 0;
        for (int i = 0; i < cnt; ++i) {
          const int blk = __shfl_sync(0xffffffffu, mine, i);
          if (lane == 0) {
            if (static_cast<unsigned long long>(static_cast<long long>(blk)) >=
                static_cast<unsigned long long>(p.num_blocks))
              atomicOr(&g_deverr_attn, AEG_DEVERR_BLOCK_ID_RANGE);  // TMA zero-fills it
            if (!abort && !mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimitNs)) {
              abort = true;
              s_flag[1] = 1;
              atomicOr(&g_deverr_attn, AEG_DEVERR_WAIT_TIMEOUT);
            }
            if (!abort) {
              uint8_t* kdst = tiles + stage * 2 * kBox;
              mbar_arrive_expect_tx(&full[stage], 2 * kBox);
              tma_load_5d(kdst, &kmap, &full[stage], 0, 0, 0, g * HG, blk, pol);
              tma_load_5d(kdst + kBox, &vmap, &full[stage], 0, 0, 0, g * HG, blk, pol);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    // Drain: make sure no bulk copy into this CTA's shared memory is still in flight at exit.
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) {
        // The last phase issued on stage s has parity (phase of its last use); waiting on
        // the empty barrier of each stage means the consumers finished (or gave up).
        if (!abort && !mbar_wait_bounded(&empty[stage], phase ^ 1, kWaitLimitNs)) {
          abort = true;
          atomicOr(&g_deverr_attn, AEG_DEVERR_WAIT_TIMEOUT);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;
  }

  // --------------------------------- consumer warps ------------------------------------
  using Mma = MmaF32<T>;
  const T* q = static_cast<const T*>(p.q);
  T* out = static_cast<T*>(p.out);
  const int lr = lane & 7;       // row within an 8x8 matrix
  const int lm = lane >> 3;      // which of the four matrices this lane addresses
  const int quad = lane & 3;     // column pair of the accumulator fragment
  const int grp = lane >> 2;     // row of the accumulator fragment
  const int cap = p.table_stride * kBlockTokens;
  const int hgG = HG * G;

  uint32_t stage = 0, phase = 0;
  for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
    const int4 un = p.ws.units[u];
    if (!unit_ok(un, u, p)) continue;
    const int pair = un.x;
    const int b = pair / NG, g = pair % NG;
    const int split = un.w >> 16, nsplit = un.w & 0xffff;
    const int kvh = g * HG + warp;
    const int n_ctx = min(max(p.seq_lens[b], 0), cap);

    // Query fragments (B operand of S^T = K Q^T): Q[head][d] with d contiguous.
    uint32_t qf[NT][8][2];
    const T* qb = q + static_cast<int64_t>(b) * p.q_stride + static_cast<int64_t>(kvh) * G * kHeadDim;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int head = nt * 8 + grp;
      const bool valid = head < G;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int d = ks * 16 + 2 * quad;
        qf[nt][ks][0] = valid ? *reinterpret_cast<const uint32_t*>(qb + head * kHeadDim + d) : 0u;
        qf[nt][ks][1] = valid ? *reinterpret_cast<const uint32_t*>(qb + head * kHeadDim + d + 8) : 0u;
      }
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

    for (int j = un.y; j < un.z; ++j) {
      bool ok = true;
      if (s_flag[1]) {
        ok = false;
      } else if (!mbar_wait_bounded(&full[stage], phase, kWaitLimitNs)) {
        ok = false;
        s_flag[1] = 1;
        if (lane == 0) atomicOr(&g_deverr_attn, AEG_DEVERR_WAIT_TIMEOUT);
      }
      const int nvalid = min(kBlockTokens, n_ctx - j * kBlockTokens);
      if (ok && nvalid > 0) {
        const uint32_t kbase = smem_u32(tiles + stage * 2 * kBox) + warp * kHeadBytes;
        const uint32_t vbase = kbase + kBox;

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
          pb[nt][0] = movmatrix_trans(pack2<T>(p0, p1));
          pb[nt][1] = movmatrix_trans(pack2<T>(p2, p3));
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
          for (int nt = 0; nt < NT; ++nt) Mma::run(o[mt][nt], a, pb[nt][0], pb[nt][1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }

    // Row sums: each lane holds the sum over its own tokens.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        l[nt][0] += __shfl_xor_sync(0xffffffffu, l[nt][0], off);
        l[nt][1] += __shfl_xor_sync(0xffffffffu, l[nt][1], off);
      }

    if (nsplit == 1) {
      T* ob = out + static_cast<int64_t>(b) * p.out_stride + static_cast<int64_t>(kvh) * G * kHeadDim;
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
      continue;
    }

    // Split unit: write fp32 partials, then take a ticket; the last split merges.
    {
      const int64_t base_hl = static_cast<int64_t>(u) * hgG + warp * G;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h0 = nt * 8 + 2 * quad;
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
          const int d0 = mt * 16 + grp;
          if (h0 < G) {
            float* po = p.ws.part_o + (base_hl + h0) * kHeadDim;
            po[d0] = o[mt][nt][0];
            po[d0 + 8] = o[mt][nt][2];
          }
          if (h0 + 1 < G) {
            float* po = p.ws.part_o + (base_hl + h0 + 1) * kHeadDim;
            po[d0] = o[mt][nt][1];
            po[d0 + 8] = o[mt][nt][3];
          }
        }
        if (grp == 0) {
          if (h0 < G) p.ws.part_ml[base_hl + h0] = make_float2(m[nt][0], l[nt][0]);
          if (h0 + 1 < G) p.ws.part_ml[base_hl + h0 + 1] = make_float2(m[nt][1], l[nt][1]);
        }
      }
    }
    __threadfence();
    named_bar(1, NCONS);
    if (threadIdx.x == 0) {
      const int old = atomicAdd(&p.ws.counters[pair], 1);
      s_flag[0] = (old == nsplit - 1) ? 1 : 0;
    }
    named_bar(1, NCONS);
    if (s_flag[0]) {
      __threadfence();
      const int first = u - split;
      for (int hl = threadIdx.x; hl < hgG; hl += NCONS) {
        float mx = -INFINITY;
        for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, __ldcg(&p.ws.part_ml[static_cast<int64_t>(first + s) * hgG + hl]).x);
        float lsum = 0.f;
        if (mx != -INFINITY)
          for (int s = 0; s < nsplit; ++s) {
            const float2 ml = __ldcg(&p.ws.part_ml[static_cast<int64_t>(first + s) * hgG + hl]);
            lsum += ex2(ml.x - mx) * ml.y;
          }
        s_mx[hl] = mx;
        s_inv[hl] = lsum > 0.f ? 1.f / lsum : 0.f;
      }
      named_bar(1, NCONS);
      T* ob = out + static_cast<int64_t>(b) * p.out_stride + static_cast<int64_t>(g) * hgG * kHeadDim;
      for (int idx = threadIdx.x; idx < hgG * kHeadDim; idx += NCONS) {
        const int hl = idx / kHeadDim;
        const int d = idx - hl * kHeadDim;
        const float mx = s_mx[hl];
        float acc = 0.f;
        if (mx != -INFINITY)
          for (int s = 0; s < nsplit; ++s) {
            const int64_t r = static_cast<int64_t>(first + s) * hgG + hl;
            acc += ex2(__ldcg(&p.ws.part_ml[r]).x - mx) * __ldcg(&p.ws.part_o[r * kHeadDim + d]);
          }
        ob[hl * kHeadDim + d] = from_float<T>(acc * s_inv[hl]);
      }
      if (threadIdx.x == 0) {
        p.ws.counters[pair] = 0;
        s_flag[0] = 0;
      }
      named_bar(1, NCONS);
    }
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
int encode_kv_map(CUtensorMap* map, const void* base, int dtype, int Hkv, int64_t block_stride, int64_t num_blocks,
                  int hg) {
  auto fn = get_encode_fn();
  if (!fn) return set_error(AEG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const cuuint64_t es = 2;
  cuuint64_t dims[5] = {64, 16, static_cast<cuuint64_t>(kHalves), static_cast<cuuint64_t>(Hkv),
                        static_cast<cuuint64_t>(num_blocks)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(Hkv) * kHeadDim * es, 64 * es, kHeadDim * es,
                           static_cast<cuuint64_t>(block_stride) * es};
  cuuint32_t box[5] = {64, 16, static_cast<cuuint32_t>(kHalves), static_cast<cuuint32_t>(hg), 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dtype == AEG_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AEG_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return AEG_OK;
}

template <typename T, int HG, int NT>
int launch_attn_t(const CUtensorMap& km, const CUtensorMap& vm, const AttnParams& prm, cudaStream_t stream) {
  auto kern = decode_attn_kernel<T, HG, NT>;
  constexpr size_t smem = attn_smem_bytes<HG>();
  // Per-device one-time set-up (kept out of the launch path so that launches can be captured
  // into CUDA graphs without further runtime configuration calls).
  constexpr int kMaxDevices = 64;
  static int per_sm_cache[kMaxDevices] = {0};
  static std::mutex mu;
  int dev = 0;
  AEG_CHECK_CUDA(cudaGetDevice(&dev));
  AEG_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "decode: device ordinal %d out of range", dev);
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (per_sm_cache[dev] == 0) {
      AEG_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
      int n = 0;
      AEG_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, (HG + 1) * 32, smem));
      per_sm_cache[dev] = n > 0 ? n : -1;
    }
    per_sm = per_sm_cache[dev];
  }
  if (per_sm < 1) return set_error(AEG_ERR_UNSUPPORTED, "decode attention kernel does not fit on an SM");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(num_sms() * per_sm));
  cfg.blockDim = dim3((HG + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  AEG_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, km, vm, prm));
  return AEG_OK;
}

template <typename T>
int launch_attn_dtype(int hg, int nt, const CUtensorMap& km, const CUtensorMap& vm, const AttnParams& prm,
                      cudaStream_t s) {
  if (hg == 4) return nt == 1 ? launch_attn_t<T, 4, 1>(km, vm, prm, s) : launch_attn_t<T, 4, 2>(km, vm, prm, s);
  if (hg == 2) return nt == 1 ? launch_attn_t<T, 2, 1>(km, vm, prm, s) : launch_attn_t<T, 2, 2>(km, vm, prm, s);
  return nt == 1 ? launch_attn_t<T, 1, 1>(km, vm, prm, s) : launch_attn_t<T, 1, 2>(km, vm, prm, s);
}

int ctas_per_sm_for(int hg) {
  // Resident CTAs per SM of the attention kernel, bounded by its shared memory ring.
  const size_t smem = hg == 4 ? attn_smem_bytes<4>() : (hg == 2 ? attn_smem_bytes<2>() : attn_smem_bytes<1>());
  int per = static_cast<int>((228 * 1024) / (smem + 1024));
  return per < 1 ? 1 : per;
}

int validate_shape(int B, int Hq, int Hkv, int D, int table_stride) {
  AEG_CHECK_ARG(B >= 0, "decode: negative batch");
  AEG_CHECK_ARG(Hkv > 0 && Hq > 0 && Hq % Hkv == 0, "decode: Hq (%d) must be a positive multiple of Hkv (%d)", Hq, Hkv);
  AEG_CHECK_ARG(Hq / Hkv <= 16, "decode: GQA group Hq/Hkv = %d exceeds 16", Hq / Hkv);
  if (D != kHeadDim) return set_error(AEG_ERR_UNSUPPORTED, "decode: head_dim %d not supported (only 128)", D);
  AEG_CHECK_ARG(table_stride > 0, "decode: block-table stride must be positive");
  AEG_CHECK_ARG(static_cast<int64_t>(B) * (Hkv / pick_hg(Hkv)) < (1 << 30), "decode: batch too large");
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

int aeg_decode_plan(void* workspace, size_t workspace_bytes, const int32_t* seq_lens, int B, int Hq, int Hkv, int D,
                    int table_stride, void* stream) {
  int st = aeg::validate_shape(B, Hq, Hkv, D, table_stride);
  if (st != AEG_OK) return st;
  AEG_CHECK_ARG(workspace != nullptr && aeg::aligned(workspace, 256), "decode_plan: workspace must be 256-byte aligned");
  const aeg::WsLayout L = aeg::ws_layout(B, Hq, Hkv, D);
  AEG_CHECK_ARG(workspace_bytes >= L.total, "decode_plan: workspace of %zu bytes, need %zu", workspace_bytes, L.total);
  AEG_CHECK_ARG(B == 0 || seq_lens != nullptr, "decode_plan: seq_lens is NULL");
  const int hg = aeg::pick_hg(Hkv);
  const int ng = Hkv / hg;
  int target = aeg::num_sms() * aeg::ctas_per_sm_for(hg);
  if (const char* e = std::getenv("AEG_DECODE_UNITS_PER_CTA")) {
    const int k = std::atoi(e);
    if (k > 0) target *= k;
  }
  if (target > aeg::kMaxTargetUnits) target = aeg::kMaxTargetUnits;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  aeg::WsPtrs w = aeg::ws_ptrs(workspace, L);
  aeg::decode_plan_kernel<<<1, aeg::kPlanThreads, 0, s>>>(seq_lens, B, ng, table_stride, target, w);
  AEG_CHECK_LAUNCH("decode_plan");
  return AEG_OK;
}

int aeg_paged_attn_decode(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k_cache,
                          const void* v_cache, int64_t block_stride, int64_t num_blocks, const int32_t* block_tables,
                          int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale,
                          int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  int st = aeg::validate_shape(B, Hq, Hkv, D, table_stride);
  if (st != AEG_OK) return st;
  if (B == 0) return AEG_OK;
  AEG_CHECK_ARG(dtype == AEG_DTYPE_FP16 || dtype == AEG_DTYPE_BF16, "decode: dtype %d is not fp16/bf16", dtype);
  AEG_CHECK_ARG(out && q && k_cache && v_cache && block_tables && seq_lens, "decode: null pointer");
  AEG_CHECK_ARG(workspace != nullptr && aeg::aligned(workspace, 256), "decode: workspace must be 256-byte aligned");
  const aeg::WsLayout L = aeg::ws_layout(B, Hq, Hkv, D);
  AEG_CHECK_ARG(workspace_bytes >= L.total, "decode: workspace of %zu bytes, need %zu", workspace_bytes, L.total);
  AEG_CHECK_ARG(num_blocks > 0 && num_blocks <= 0x7fffffffLL, "decode: num_blocks %lld out of range", (long long)num_blocks);
  AEG_CHECK_ARG(aeg::aligned(k_cache, 16) && aeg::aligned(v_cache, 16), "decode: K/V cache bases must be 16-byte aligned");
  AEG_CHECK_ARG(block_stride % 8 == 0 && block_stride >= int64_t(16) * Hkv * D,
                "decode: block stride %lld must be a multiple of 8 elements and >= 16*Hkv*D", (long long)block_stride);
  AEG_CHECK_ARG(q_stride >= int64_t(Hq) * D && out_stride >= int64_t(Hq) * D, "decode: q/out token stride < Hq*D");
  AEG_CHECK_ARG(aeg::aligned(q, 4) && q_stride % 2 == 0, "decode: q must be 4-byte aligned with an even token stride");
  AEG_CHECK_ARG(aeg::aligned(out, 2), "decode: out must be 2-byte aligned");
  AEG_CHECK_ARG(aeg::aligned(block_tables, 4) && aeg::aligned(seq_lens, 4), "decode: int32 arrays must be aligned");

  const int hg = aeg::pick_hg(Hkv);
  CUtensorMap km, vm;
  st = aeg::encode_kv_map(&km, k_cache, dtype, Hkv, block_stride, num_blocks, hg);
  if (st != AEG_OK) return st;
  st = aeg::encode_kv_map(&vm, v_cache, dtype, Hkv, block_stride, num_blocks, hg);
  if (st != AEG_OK) return st;

  aeg::AttnParams prm{};
  prm.out = out;
  prm.out_stride = out_stride;
  prm.q = q;
  prm.q_stride = q_stride;
  prm.tables = block_tables;
  prm.table_stride = table_stride;
  prm.seq_lens = seq_lens;
  prm.G = Hq / Hkv;
  prm.NG = Hkv / hg;
  prm.num_pairs = B * prm.NG;
  prm.max_units = L.max_units;
  prm.num_blocks = num_blocks;
  prm.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);  // log2(e)
  prm.ws = aeg::ws_ptrs(workspace, L);
  const int nt = prm.G <= 8 ? 1 : 2;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AEG_DTYPE_BF16) return aeg::launch_attn_dtype<__nv_bfloat16>(hg, nt, km, vm, prm, s);
  return aeg::launch_attn_dtype<__half>(hg, nt, km, vm, prm, s);
}

}  // extern "C"
