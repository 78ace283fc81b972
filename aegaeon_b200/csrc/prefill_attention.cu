// Prefill (prompt) attention: causal attention of each prompt's tokens over the prompt itself,
// varlen batch, GQA.
//
// Reference: vLLM 0.5.1's FlashAttention backend runs prompts (no chunked prefill in Aegaeon,
// aegaeon/aegaeon/worker.py:603-609, 619-626) through
// `flash_attn_varlen_func(q, k, v, cu_seqlens_q=query_start_loc, cu_seqlens_k=seq_start_loc,
// max_seqlen_q, max_seqlen_k, softmax_scale, causal=True)` on the prompt tokens' q/k/v (the paged
// cache is written by reshape_and_cache alongside). Query token i of a prompt sees keys 0..i of
// the same prompt; query head h reads KV head h / (Hq / Hkv).
//
// The kernel runs on the 5th-generation tensor cores (tcgen05.mma with TMEM accumulators, operands
// staged by TMA); its structure is described below. Query tiles are visited heaviest first (the
// last query tile of a prompt sees the most keys). Measured and rejected: an mma.sync kernel (64
// rows per CTA, cp.async double buffering; fp16 206 / bf16 163 TFLOP/s on the bench prompts), a
// serialized tcgen05 kernel (one 128-row tile, O folded into registers every key tile: 171 / 139),
// a mask-free softmax path for fully visible key tiles (a branch around the warp-collective TMEM
// loads: 0.414 vs 0.316 ms), one thread issuing every load and MMA with P through shared memory
// (284 / 328: a refill waited for all MMAs of the previous key tile before the next P was
// served), one MMA thread serving both query tiles in the order their P arrive (312 / 360 with
// one thread vs 357 / 409 with one per query tile: issuing a tile's P V and next scores takes
// that thread 0.5-0.6 us), one CTA per item (357 / 409 vs 391 / 488 persistent: per CTA ~0.7 us
// of setup, ~2 us before the first scores and ~1 us between CTAs on an SM), and 16-byte output
// stores straight from each lane's row (32 rows touched per store instruction: the epilogue took
// ~2 us, most of it waiting on those stores), items of two consecutive row tiles of one head
// for every head (tile B then needs two more key tiles than A, which waits: 402 / 505 vs 434 /
// 516 with head pairs), and 2, 3 or 4 of every 8 exponents taken on the
// FMA pipe by range reduction and a polynomial instead of ex2 (bf16 / fp16 338 / 432, 335 / 423,
// 303 / 398 vs 391 / 488: the softmax is bound by instruction issue, not by the ex2 unit).
#include "aeg_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <type_traits>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_prefill = 0;

constexpr int kPD = 128;  // head dim

__device__ __forceinline__ float ex2p(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Two fp32 lanes in one instruction (sm_100 packed f32x2): a * b + c, and a + b.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// ---------------------------------------------------------------------------------------
// tcgen05 kernel, persistent: one CTA per SM works through items taken from a per-launch counter.
// An item is two 128-row query tiles A and B of one prompt whose heads share a KV head: the same
// rows of two query heads (GQA), or, for a lone head, two consecutive row tiles of it. Each tile
// is owned by a softmax warpgroup (warps 0-3 and 4-7; thread t of a warpgroup owns query row t of
// its tile = TMEM lane t); each tile has an MMA warp (warps 8 and 10) whose first thread issues its
// tcgen05.mma, and a load warp (warp 9) whose first thread fetches items and issues every TMA
// load. Keys come in tiles of 64 through a 4-stage TMA ring shared by both query tiles and
// running on across items; the load thread refills a stage as soon as the MMAs that read it have
// completed, and publishes the next item's record and Q as soon as every warp is done with the
// current ones. Per key tile j and query tile X:
//   S_X(j) = Q_X K(j)^T  8 MMAs (M 128, N 64, K 16) into TMEM S_X[j & 1] (64 fp32 columns);
//   softmax               the warpgroup reads its rows of S_X(j) in one tcgen05.ld, computes
//                         exp2 / sum, and writes P in the input dtype back over S_X(j) in TMEM
//                         (32 columns of b16 pairs; bf16: its rounding residue in the other 32);
//   O_X += P V(j)          4 MMAs (M 128, N 128, K 16; bf16: 8) into TMEM O_X with A = P read from
//                         TMEM and B = V read MN-major straight from its TMA layout.
// MMAs issued by one thread run in issue order, so S_X(j + 2), issued after O_X += P V(j), cannot
// overwrite P_X(j) before it is read. O never leaves TMEM until the item's epilogue: a row is
// rescaled in place (tcgen05.ld / st) only when its running maximum grows by more than 8 in the
// exp2 domain, so P stays below 2^8, and only then does the softmax wait for the previous P V.
// While one warpgroup runs its softmax the tensor pipe works on the other tile's MMAs. Every wait
// is bounded: a timeout is recorded, the CTA stops issuing, drains its own loads and MMAs
// (bounded), frees TMEM and returns; rows it did not finish are not written.
constexpr int kTM = 128;                 // query rows per tile (two tiles per item)
constexpr int kTN = 64;                  // keys per tile
constexpr int kTThreads = 11 * 32;       // 2 softmax warpgroups, the MMA warps of tiles A and B, the load warp
constexpr int kQHalf = kTM * 128;        // one SW128 box of Q: 128 rows x 64 elements (16 KiB)
constexpr int kKHalf = kTN * 128;        // one SW128 box of K or V: 64 rows x 64 elements (8 KiB)
constexpr uint32_t kTmemCols = 512;      // S_A[2], S_B[2] (64 each), O_A, O_B (128 each)
constexpr uint64_t kTcWaitNs = 2000000000ull;
constexpr float kRescaleAbove = 8.f;     // exp2 domain

// Shared-memory layout: Q_A and Q_B, the K and V stages, and a 4 KiB output staging tile per
// softmax warp (P lives in TMEM).
struct TcLayout {
  static constexpr int kStages = 4;
  static constexpr int kOffQ = 0;                                   // Q_A, Q_B: 2 halves each
  static constexpr int kOffK = kOffQ + 4 * kQHalf;                  // stage s: 2 halves
  static constexpr int kOffV = kOffK + kStages * 2 * kKHalf;        // stage s: 2 halves
  static constexpr int kOffE = kOffV + kStages * 2 * kKHalf;        // warp w: 32 rows x 128 bytes
  static constexpr int kOffBar = kOffE + 8 * 4096;
  static constexpr int kSmem = kOffBar + 512 + 1024;                // + 1024-byte alignment slack
};
static_assert(TcLayout::kSmem <= 232448, "prefill smem above the 227 KB per-CTA limit");

// mbarrier slots. QFull: the item record and its Q landed; QFree: every warp is done with them
// (both MMA threads after their last S, each softmax warp after reading the record).
constexpr int kBarQFull = 0, kBarQFree = 1, kBarKFull = 2, kBarVFull = kBarKFull + TcLayout::kStages,
              kBarKFree = kBarVFull + TcLayout::kStages, kBarVFree = kBarKFree + TcLayout::kStages,
              kBarSFull = kBarVFree + TcLayout::kStages,  // S: [X][buf]
    kBarPFull = kBarSFull + 4, kBarPv = kBarPFull + 2, kBarOFree = kBarPv + 2, kBarDrain = kBarOFree + 2,
              kBarCount = kBarDrain + 2;
constexpr int kQFreeArrivals = 2 + 8;

// One work item of the prompt at s0 of length L: query tile A (128 rows from qA of head hA) and
// query tile B (128 rows from qB of head hB; none when nB = 0), with nA / nB key tiles; both
// heads read the same KV head. nA < 0 marks the end of the work.
struct PfItem {
  int s0, L, qA, qB, hA, hB, nA, nB;
};
static_assert(8 * kBarCount + 8 + sizeof(PfItem) <= 512,
              "mbarrier slots, the TMEM address, the abort flag and the item record fit the barrier area");

// Work counters: each launch takes one of kCounterSlots (round robin on the host), its CTAs take
// items with atomicAdd, and the last CTA to run out of work sets both back to zero.
constexpr int kCounterSlots = 64;
__device__ unsigned int g_pf_next[kCounterSlots];
__device__ unsigned int g_pf_done[kCounterSlots];

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// SW128 smem matrix descriptor (version 1): start >> 4, LBO >> 4, SBO >> 4, layout type 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16, fp32 accumulator, M = 128, A K-major.
template <typename T>
__device__ __forceinline__ uint32_t idesc_f16(int n, bool b_mn_major) {
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(n) >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// The same with A read from TMEM (K-major: row i in lane i, two 16-bit elements per column).
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Non-blocking probe of an mbarrier phase (mbarrier.test_wait returns at once).
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// OR of `v` over the 128 threads of named barrier `id` (a barrier itself: every thread must come).
__device__ __forceinline__ bool group_any(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, %2, 128, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}


__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// 32 fp32 columns of this thread's TMEM lane, load and wait in one statement.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// The 64 fp32 columns of this thread's TMEM lane starting at `taddr`, in one round trip: the load
// and its wait are one statement, so no use of the registers can be placed before the wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

template <typename T>
__global__ void __launch_bounds__(kTThreads, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                  const __grid_constant__ CUtensorMap vmap, T* __restrict__ out, int64_t o_stride,
                  const int32_t* __restrict__ cu_seqlens, int64_t num_tokens, int B, int Hq, int levels,
                  int max_seqlen, int G, float scale_log2, int slot) {
  constexpr bool kSplitP = std::is_same<T, __nv_bfloat16>::value;  // P as value + rounding residue
  using LY = TcLayout;
  constexpr int kSt = LY::kStages;
  extern __shared__ uint8_t tsmem_raw[];
  const uint32_t raw = smem_u32(tsmem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* smem = tsmem_raw + (base - raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LY::kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + LY::kOffBar + 8 * kBarCount);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + LY::kOffBar + 8 * kBarCount + 4);  // a wait gave up
  volatile PfItem* s_item = reinterpret_cast<volatile PfItem*>(smem + LY::kOffBar + 8 * kBarCount + 8);
  auto bar_u32 = [&](int i) { return base + LY::kOffBar + 8u * static_cast<uint32_t>(i); };
  const int tid = threadIdx.x, warp = tid >> 5;

  if (tid == 0) {
    for (int i = 0; i < kBarCount; ++i) mbar_init(&bars[i], 1);
    mbar_init(&bars[kBarQFree], kQFreeArrivals);
    for (int i = 0; i < kSt; ++i) {  // a stage is released by both query tiles' MMA threads
      mbar_init(&bars[kBarKFree + i], 2);
      mbar_init(&bars[kBarVFree + i], 2);
    }
    fence_mbar_init();
    *s_abort = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto tmem_s = [&](int x, int buf) { return tmem + static_cast<uint32_t>((x * 2 + buf) * 64); };
  auto tmem_o = [&](int x) { return tmem + 256u + static_cast<uint32_t>(x) * 128u; };
  const uint32_t sQ = base + LY::kOffQ;
  auto sQx = [&](int x) { return sQ + static_cast<uint32_t>(x) * 2 * kQHalf; };
  auto sK = [&](int st) { return base + LY::kOffK + static_cast<uint32_t>(st) * 2 * kKHalf; };
  auto sV = [&](int st) { return base + LY::kOffV + static_cast<uint32_t>(st) * 2 * kKHalf; };

  bool abort = false;
  if (warp == 9) {
    // ------------------------------- work items and loads -------------------------------
    // The counter runs over (level of 256 query rows, prompt, head slot), heaviest level first;
    // a (level, prompt) has Hq slots, G per KV head. With G >= 2 a KV head's first 2 * (G / 2)
    // slots are head pairs (2p, 2p + 1) over the later 128 rows of the level, then over the
    // earlier 128: both tiles of such an item have the same rows, so they need the same key
    // tiles and share them. An odd G's last head takes the level's two 128-row tiles as A and B
    // (B then needs two more key tiles than A), as does every head when G = 1. The next item is
    // fetched while the current one computes; its Q and the item record go out once every warp is
    // done with the current item's (QFree), its key tiles into the ring as the MMA threads
    // release stages.
    if ((tid & 31) == 0) {
      const unsigned per_level = static_cast<unsigned>(B) * static_cast<unsigned>(Hq);
      const unsigned total = per_level * static_cast<unsigned>(levels);
      auto fetch = [&](PfItem& it) {
        it.nA = -1;
        while (!*s_abort) {
          const unsigned i = atomicAdd(&g_pf_next[slot], 1u);
          if (i >= total) return;
          const int lv = static_cast<int>(i / per_level);
          const int rem = static_cast<int>(i % per_level);
          const int b = rem / Hq, slot_h = rem % Hq;
          const int lv0 = (levels - 1 - lv) * 2 * kTM;  // first row of the level
          const int s0 = cu_seqlens[b];
          const int L = cu_seqlens[b + 1] - s0;
          const bool valid = s0 >= 0 && L >= 0 && static_cast<int64_t>(s0) + L <= num_tokens && L <= max_seqlen;
          if (!valid) atomicOr(&g_deverr_prefill, AEG_DEVERR_SEQ_LEN_RANGE);
          if (!valid || L == 0 || lv0 >= L) {
            // every slot of this (level, prompt) is empty: move the counter past them
            atomicMax(&g_pf_next[slot], static_cast<unsigned>(lv) * per_level + static_cast<unsigned>(b + 1) * Hq);
            continue;
          }
          const int kvh = slot_h / G, j = slot_h % G, pairs = G / 2;
          it.s0 = s0;
          it.L = L;
          if (j < 2 * pairs) {  // heads (2p, 2p + 1) of the KV head, one 128-row half of the level
            const int q0 = lv0 + (j < pairs ? kTM : 0);
            if (q0 >= L) continue;
            it.qA = it.qB = q0;
            it.hA = kvh * G + 2 * (j % pairs);
            it.hB = it.hA + 1;
            it.nA = it.nB = (min(L, q0 + kTM) + kTN - 1) / kTN;
          } else {  // the last head of an odd G: the level's two 128-row tiles
            it.qA = lv0;
            it.qB = lv0 + kTM;
            it.hA = it.hB = kvh * G + G - 1;
            it.nA = (min(L, lv0 + kTM) + kTN - 1) / kTN;
            it.nB = lv0 + kTM < L ? (min(L, lv0 + 2 * kTM) + kTN - 1) / kTN : 0;
          }
          return;
        }
      };
      // One polling loop: the next item's record and Q go out as soon as every warp is done with
      // the previous ones (its tiles are issued by then: the last S of an item reads its last
      // key tile), and key tiles are issued in ring order as stages come free. The item after
      // that is fetched right after a publication, while the current one computes.
      PfItem nxt;
      fetch(nxt);
      // Published items whose key tiles are not all issued: at most two (an item is published
      // only after the previous one's last key tile has landed), the older in p0.
      struct Pending {
        int g0, n, s0, kvh;
      } p0{0, 0, 0, 0}, p1{0, 0, 0, 0};
      int n_pend = 0;
      int k = 0;              // items published
      int t_next = 0;         // key tiles issued so far (over all items)
      int t_end = 0;          // key tiles of the published items
      bool published_end = false;
      bool ok = true;
      uint64_t idle_since = 0;
      while (ok && !(published_end && t_next == t_end)) {
        bool progressed = false;
        if (!published_end && (k == 0 || mbar_test(&bars[kBarQFree], static_cast<uint32_t>((k - 1) & 1)))) {
          s_item->s0 = nxt.s0;
          s_item->L = nxt.L;
          s_item->qA = nxt.qA;
          s_item->qB = nxt.qB;
          s_item->hA = nxt.hA;
          s_item->hB = nxt.hB;
          s_item->nA = nxt.nA;
          s_item->nB = nxt.nB;
          if (nxt.nA < 0) {  // no more work: the record alone
            mbar_arrive(&bars[kBarQFull]);
            published_end = true;
          } else {
            const PfItem it = nxt;
            const int n_tiles = max(it.nA, it.nB);
            mbar_arrive_expect_tx(&bars[kBarQFull], (it.nB > 0 ? 4 : 2) * kQHalf);
            tma_load_2d(sQx(0), &qmap, bar_u32(kBarQFull), it.hA * 128, it.s0 + it.qA);
            tma_load_2d(sQx(0) + kQHalf, &qmap, bar_u32(kBarQFull), it.hA * 128 + 64, it.s0 + it.qA);
            if (it.nB > 0) {
              tma_load_2d(sQx(1), &qmap, bar_u32(kBarQFull), it.hB * 128, it.s0 + it.qB);
              tma_load_2d(sQx(1) + kQHalf, &qmap, bar_u32(kBarQFull), it.hB * 128 + 64, it.s0 + it.qB);
            }
            (n_pend == 0 ? p0 : p1) = Pending{t_end, n_tiles, it.s0, it.hA / G};
            ++n_pend;
            t_end += n_tiles;
            ++k;
            fetch(nxt);
          }
          progressed = true;
        }
        if (t_next < t_end) {
          const int g = t_next;  // global tile g into stage g % kSt, after tile g - kSt's release
          const uint32_t pph = static_cast<uint32_t>(((g - kSt) / kSt) & 1);
          if (g < kSt || (mbar_test(&bars[kBarKFree + g % kSt], pph) && mbar_test(&bars[kBarVFree + g % kSt], pph))) {
            const Pending pi = p0;
            const int st = g % kSt, y = pi.s0 + (g - pi.g0) * kTN, xc = pi.kvh * 128;
            mbar_arrive_expect_tx(&bars[kBarKFull + st], 2 * kKHalf);
            tma_load_2d(sK(st), &kmap, bar_u32(kBarKFull + st), xc, y);
            tma_load_2d(sK(st) + kKHalf, &kmap, bar_u32(kBarKFull + st), xc + 64, y);
            mbar_arrive_expect_tx(&bars[kBarVFull + st], 2 * kKHalf);
            tma_load_2d(sV(st), &vmap, bar_u32(kBarVFull + st), xc, y);
            tma_load_2d(sV(st) + kKHalf, &vmap, bar_u32(kBarVFull + st), xc + 64, y);
            ++t_next;
            if (t_next == pi.g0 + pi.n) {
              p0 = p1;
              --n_pend;
            }
            progressed = true;
          }
        }
        if (progressed) {
          idle_since = 0;
        } else {
          const uint64_t now = globaltimer_ns();
          if (idle_since == 0) idle_since = now;
          if (now - idle_since > kTcWaitNs || *s_abort) ok = false;
        }
      }
      if (!ok && k > 0 && !published_end) {
        // the last published item's Q may still be in flight: it lands before the CTA exits
        mbar_wait_bounded(&bars[kBarQFull], static_cast<uint32_t>((k - 1) & 1), kTcWaitNs);
      }
      // The launch's counter goes back to zero once every CTA has run out of work.
      __threadfence();
      if (atomicAdd(&g_pf_done[slot], 1u) == gridDim.x - 1) {
        atomicExch(&g_pf_next[slot], 0u);
        atomicExch(&g_pf_done[slot], 0u);
      }
      // The last kSt key tiles may still be in flight (earlier ones were consumed before their
      // stage was reused): they land before the CTA exits, bounded.
      for (int g = max(0, t_next - kSt); g < t_next; ++g) {
        const uint32_t ph = static_cast<uint32_t>((g / kSt) & 1);
        if (!mbar_wait_bounded(&bars[kBarKFull + g % kSt], ph, kTcWaitNs)) ok = false;
        if (!mbar_wait_bounded(&bars[kBarVFull + g % kSt], ph, kTcWaitNs)) ok = false;
      }
      if (!ok) {
        *s_abort = 1;
        __threadfence_block();
      }
      abort = !ok;
    }
  } else if (warp == 8 || warp == 10) {
    // ------------------------------- MMA issue, query tile x -------------------------------
    // Each query tile has its own MMA thread (warps 8 and 10 sit on different SM sub-partitions),
    // so the two tiles' MMAs are issued in parallel and neither waits behind the other. Per item,
    // the scores run two key tiles ahead of the softmax: S_x(0) and S_x(1) first, then, as soon
    // as softmax x has published P_x(j), O_x += P_x V(j) and the scores S_x(j + 2) into the
    // buffer that P_x(j) occupies (the P V ahead of it in this thread's issue order has read
    // P_x(j) by then). The first P V of an item waits until softmax x has read O_x out for the
    // previous item. A key tile's stage goes back to the load thread after two arrivals: one
    // commit per query tile that reads it, and a plain arrival from the tile's MMA thread for a
    // query tile that does not. Sequence numbers run over all items: gx counts this tile's key
    // tiles (S buffer gx & 1, barrier phases), ex its items, t_base the ring's tiles.
    const int x = warp == 8 ? 0 : 1;
    if ((tid & 31) == 0) {
      const uint32_t id_s = idesc_f16<T>(kTN, false), id_o = idesc_f16<T>(128, true);
      bool ok = true;
      auto wait_kv = [&](int base_bar, int t) {
        ok = ok && !*s_abort &&
             mbar_wait_bounded(&bars[base_bar + t % kSt], static_cast<uint32_t>((t / kSt) & 1), kTcWaitNs);
      };
      // S of sequence number g into S_x[g & 1] from ring tile tg. That buffer last held P of
      // sequence g - 2, read by the P V this thread issued just before.
      auto issue_s = [&](int g, int tg) {
        const int st = tg % kSt;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t qo = static_cast<uint32_t>(kk >> 2) * kQHalf + static_cast<uint32_t>(kk & 3) * 32;
          const uint32_t ko = static_cast<uint32_t>(kk >> 2) * kKHalf + static_cast<uint32_t>(kk & 3) * 32;
          umma_f16(tmem_s(x, g & 1), sw128_desc(sQx(x) + qo, 16, 1024), sw128_desc(sK(st) + ko, 16, 1024), id_s,
                   kk > 0);
        }
        umma_commit(bar_u32(kBarSFull + x * 2 + (g & 1)));
      };
      int t_base = 0, gx = 0, ex = 0;
      for (int k = 0; ok; ++k) {
        ok = !*s_abort && mbar_wait_bounded(&bars[kBarQFull], static_cast<uint32_t>(k & 1), kTcWaitNs);
        if (!ok) break;
        const int nA = s_item->nA, nB = s_item->nB;
        if (nA < 0) break;
        const int nx = x == 0 ? nA : nB;
        const int n_other = x == 0 ? nB : nA;
        const int n_tiles = max(nA, nB);
        if (nx == 0) {  // no tile x in this item
          mbar_arrive(&bars[kBarQFree]);
          t_base += n_tiles;
          continue;
        }
        for (int t = 0; t < min(2, nx) && ok; ++t) {
          wait_kv(kBarKFull, t_base + t);
          if (!ok) break;
          tc_fence_after();
          issue_s(gx + t, t_base + t);
        }
        if (!ok) break;
        if (nx <= 2) umma_commit(bar_u32(kBarQFree));  // Q_x is read by no later MMA of this item
        for (int j = 0; j < nx && ok; ++j) {
          const int g = gx + j, tg = t_base + j, st = tg % kSt;
          ok = !*s_abort && mbar_wait_bounded(&bars[kBarPFull + x], static_cast<uint32_t>(g & 1), kTcWaitNs);
          wait_kv(kBarVFull, tg);
          if (j + 2 < nx) wait_kv(kBarKFull, tg + 2);
          if (ok && j == 0 && ex > 0)
            ok = mbar_wait_bounded(&bars[kBarOFree + x], static_cast<uint32_t>((ex - 1) & 1), kTcWaitNs);
          if (!ok) break;
          tc_fence_after();
          const uint32_t pa = tmem_s(x, g & 1);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_f16_ts(tmem_o(x), pa + kk * 8, sw128_desc(sV(st) + kk * 2048, kKHalf, 1024), id_o,
                        (j > 0 || kk > 0) ? 1u : 0u);
            if constexpr (kSplitP)
              umma_f16_ts(tmem_o(x), pa + 32 + kk * 8, sw128_desc(sV(st) + kk * 2048, kKHalf, 1024), id_o, 1u);
          }
          umma_commit(bar_u32(kBarPv + x));
          if (j + 2 < nx) {
            issue_s(g + 2, tg + 2);
            if (j + 3 == nx) umma_commit(bar_u32(kBarQFree));  // that was the item's last S_x
          }
          // K(tg) was read by S_x and V(tg) by O_x += P_x V, both issued before this point
          umma_commit(bar_u32(kBarKFree + st));
          umma_commit(bar_u32(kBarVFree + st));
          if (j >= n_other) {
            mbar_arrive(&bars[kBarKFree + st]);
            mbar_arrive(&bars[kBarVFree + st]);
          }
        }
        gx += nx;
        ++ex;
        t_base += n_tiles;
      }
      // every MMA this thread issued has completed before TMEM is freed
      umma_commit(bar_u32(kBarDrain + x));
      if (!mbar_wait_bounded(&bars[kBarDrain + x], 0, kTcWaitNs)) ok = false;
      if (!ok) {
        *s_abort = 1;
        __threadfence_block();
        // release softmax x from any wait on this thread
        mbar_arrive(&bars[kBarSFull + x * 2]);
        mbar_arrive(&bars[kBarSFull + x * 2 + 1]);
        mbar_arrive(&bars[kBarPv + x]);
      }
      abort = !ok;
    }
  } else {
    // ------------------------------- softmax warpgroup x -------------------------------
    const int x = warp >> 2;
    const int r = tid & 127;  // row of the tile, TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    // tcgen05.ld / st are warp-collective (.sync.aligned): a wait's outcome is made uniform over
    // the warp before the warp acts on it. The warpgroup meets once per key tile, at the barrier
    // that publishes P, which also votes on a timeout: a warp whose wait gave up skips its work
    // but still reaches that barrier, and then all four warps stop together.
    int gx = 0;  // key tiles of this query tile over all items (S buffer and barrier phases)
    for (int k = 0; !abort; ++k) {
      bool bad = *s_abort || !mbar_wait_bounded(&bars[kBarQFull], static_cast<uint32_t>(k & 1), kTcWaitNs);
      if (group_any(1 + x, bad)) {
        abort = true;
        break;
      }
      const int s0 = s_item->s0, L = s_item->L;
      const int q0 = x == 0 ? s_item->qA : s_item->qB, h = x == 0 ? s_item->hA : s_item->hB;  // this tile's
      const int nA = s_item->nA, nB = s_item->nB;
      __syncwarp();
      if ((tid & 31) == 0) mbar_arrive(&bars[kBarQFree]);  // this warp has read the item record
      if (nA < 0) break;
      const int nx = x == 0 ? nA : nB;
      if (nx == 0) continue;
      const int row = q0 + r;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nx; ++j) {
        const int g = gx + j;
        bad = bad || *s_abort ||
              !mbar_wait_bounded(&bars[kBarSFull + x * 2 + (g & 1)], static_cast<uint32_t>((g >> 1) & 1), kTcWaitNs);
        bad = __any_sync(0xffffffffu, bad);
        // The row's 64 scores in one TMEM round trip. Keys this row cannot see become -inf; a key
        // tile that every row of the query tile sees whole (uniform over the warpgroup) needs no
        // mask. The scale is positive, so the row maximum is taken on the raw scores and scaled
        // once, and each exponent below is one fused multiply-add.
        const int key0 = j * kTN;
        float sv[64];
        float mx = -INFINITY;
        if (!bad) {
          tc_fence_after();
          tmem_ld64(tmem_s(x, g & 1) + lane_off, sv);
          if (!(key0 + kTN - 1 <= q0 && key0 + kTN <= L)) {
#pragma unroll
            for (int i = 0; i < 64; ++i) {
              const int key = key0 + i;
              sv[i] = (key <= row && key < L) ? sv[i] : -INFINITY;
            }
          }
          // a tree of 3-input maxima: 32 instructions, 4 deep
          float m1[22], m2[8];
#pragma unroll
          for (int i = 0; i < 21; ++i) m1[i] = max3f(sv[3 * i], sv[3 * i + 1], sv[3 * i + 2]);
          m1[21] = sv[63];
#pragma unroll
          for (int i = 0; i < 7; ++i) m2[i] = max3f(m1[3 * i], m1[3 * i + 1], m1[3 * i + 2]);
          m2[7] = m1[21];
          mx = max3f(max3f(m2[0], m2[1], m2[2]), max3f(m2[3], m2[4], m2[5]), fmaxf(m2[6], m2[7]));
          mx *= scale_log2;
        }
        const bool grow = mx > m_used + kRescaleAbove;
        const float factor = grow ? ex2p(m_used - mx) : 1.f;  // 0 while the row has seen nothing
        // The previous P V is waited for once per key tile, between S landing and P being
        // published: S of sequence g was issued after the P V of g - 2 and the P V of g is issued
        // only after the publication, so the barrier's pending phase is g - 1 or g and the parity
        // wait is exact. The wait also keeps this warpgroup at most one publication ahead of the
        // MMA thread. O rows are rescaled in TMEM by the whole warp when any of its rows needs it,
        // which needs that P V done first; otherwise the wait comes after the P stores.
        const bool rescale = !bad && j > 0 && __any_sync(0xffffffffu, grow && m_used != -INFINITY);
        if (rescale) {
          bad = !mbar_wait_bounded(&bars[kBarPv + x], static_cast<uint32_t>((g - 1) & 1), kTcWaitNs);
          bad = __any_sync(0xffffffffu, bad);
        }
        if (bad) {  // this warp stops working; it still meets the others below
          if (group_any(1 + x, true)) {
            abort = true;
            break;
          }
          continue;
        }
        if (rescale) {
          tc_fence_after();
          const uint32_t to = tmem_o(x) + lane_off;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float v[16];
            tmem_ld16(to + c * 16, v);
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] *= factor;
            tmem_st16(to + c * 16, v);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        if (grow) {
          l *= factor;
          m_used = mx;
        }
        const float neg_base = m_used == -INFINITY ? 0.f : -m_used;
        float2 rsum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};  // independent partial row sums
        const float2 scale2 = make_float2(scale_log2, scale_log2), base2 = make_float2(neg_base, neg_base);
        const uint32_t tp = tmem_s(x, g & 1) + lane_off;  // P over S: keys 2c, 2c + 1 in column c
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[8], pr[8];
#pragma unroll
          for (int i = 0; i < 16; i += 2) {
            const float2 a = fma2(make_float2(sv[c * 16 + i], sv[c * 16 + i + 1]), scale2, base2);
            const float p0 = ex2p(a.x), p1 = ex2p(a.y);  // masked keys: ex2(-inf) = 0
            rsum[(i >> 1) & 1] = add2(rsum[(i >> 1) & 1], make_float2(p0, p1));
            pk[i >> 1] = pack2<T>(p0, p1);
            if constexpr (kSplitP) {
              const float2 rr = unpack2<T>(pk[i >> 1]);
              pr[i >> 1] = pack2<T>(p0 - rr.x, p1 - rr.y);
            }
          }
          tmem_st8(tp + c * 8, pk);  // keys c*16 .. c*16+15
          if constexpr (kSplitP) tmem_st8(tp + 32 + c * 8, pr);
        }
        l += (rsum[0].x + rsum[1].x) + (rsum[0].y + rsum[1].y);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        bool late = false;
        if (j > 0 && !rescale) {
          late = !mbar_wait_bounded(&bars[kBarPv + x], static_cast<uint32_t>((g - 1) & 1), kTcWaitNs);
          late = __any_sync(0xffffffffu, late);
        }
        tc_fence_before();
        if (group_any(1 + x, late)) {  // P published by all four warps, unless one of them gave up
          abort = true;
          break;
        }
        if (r == 0) mbar_arrive(&bars[kBarPFull + x]);
      }
      if (abort) break;
      {
        const bool late = !mbar_wait_bounded(&bars[kBarPv + x], static_cast<uint32_t>((gx + nx - 1) & 1), kTcWaitNs) ||
                          *s_abort;
        if (group_any(1 + x, late)) {
          abort = true;
          break;
        }
      }
      tc_fence_after();
      // Epilogue: O_x / l in two TMEM round trips of 64 columns. Each warp turns its 32 rows
      // around through its 4 KiB staging tile (16-byte chunk c of row i at chunk c ^ (i & 7): no
      // bank conflicts either way), so that each global store writes four whole 128-byte row
      // segments instead of 32 pieces of 16 bytes. Rows past the prompt end are not written.
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int lane = tid & 31;
      const uint32_t stg = base + LY::kOffE + static_cast<uint32_t>(warp) * 4096u;
      const int row0 = q0 + (warp & 3) * 32;  // row of lane 0 of this warp
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int qt = 0; qt < 2; ++qt) {
          float v[32];
          tmem_ld32(tmem_o(x) + lane_off + half * 64 + qt * 32, v);
#pragma unroll
          for (int c4 = 0; c4 < 4; ++c4) {
            const int c = qt * 4 + c4;
            const uint32_t a = stg + static_cast<uint32_t>(lane) * 128u + static_cast<uint32_t>((c ^ (lane & 7)) * 16);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a),
                         "r"(pack2<T>(v[c4 * 8 + 0] * inv, v[c4 * 8 + 1] * inv)),
                         "r"(pack2<T>(v[c4 * 8 + 2] * inv, v[c4 * 8 + 3] * inv)),
                         "r"(pack2<T>(v[c4 * 8 + 4] * inv, v[c4 * 8 + 5] * inv)),
                         "r"(pack2<T>(v[c4 * 8 + 6] * inv, v[c4 * 8 + 7] * inv))
                         : "memory");
          }
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + (lane >> 3), cc = lane & 7;  // row rr of the warp, chunk cc
          const uint32_t a = stg + static_cast<uint32_t>(rr) * 128u + static_cast<uint32_t>((cc ^ (rr & 7)) * 16);
          uint4 w;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w) : "r"(a) : "memory");
          if (row0 + rr < L)
            *reinterpret_cast<uint4*>(out + static_cast<int64_t>(s0 + row0 + rr) * o_stride + static_cast<int64_t>(h) * 128 +
                                      half * 64 + cc * 8) = w;
        }
        __syncwarp();
      }
      // O_x has been read: the next item's first P V may overwrite it
      tc_fence_before();
      group_any(1 + x, false);
      if (r == 0) mbar_arrive(&bars[kBarOFree + x]);
      gx += nx;
    }
  }
  if (abort) atomicOr(&g_deverr_prefill, AEG_DEVERR_WAIT_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D map over [rows, cols] (row stride in elements), boxes of 64 elements x box_rows, 128-byte swizzle.
int encode_rows_map(CUtensorMap* map, const void* base, int dtype, int64_t rows, int64_t cols, int64_t row_stride,
                    int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(AEG_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype == AEG_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(AEG_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
  return AEG_OK;
}

template <typename T>
int launch_prefill_tc(void* out, int64_t o_stride, const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                      const void* v, int64_t v_stride, const int32_t* cu, int64_t num_tokens, int B, int max_seqlen,
                      int Hq, int Hkv, float scale, int dtype, cudaStream_t stream) {
  CUtensorMap qm, km, vm;
  int st = encode_rows_map(&qm, q, dtype, num_tokens, int64_t(Hq) * kPD, q_stride, kTM);
  if (st == AEG_OK) st = encode_rows_map(&km, k, dtype, num_tokens, int64_t(Hkv) * kPD, k_stride, kTN);
  if (st == AEG_OK) st = encode_rows_map(&vm, v, dtype, num_tokens, int64_t(Hkv) * kPD, v_stride, kTN);
  if (st != AEG_OK) return st;
  constexpr int kMaxDevices = 64;
  static bool configured[kMaxDevices] = {false};
  static std::mutex mu;
  int dev = 0;
  AEG_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(AEG_ERR_UNSUPPORTED, "prefill_attention: device %d", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      AEG_CHECK_CUDA(cudaFuncSetAttribute(prefill_tc_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         TcLayout::kSmem));
      configured[dev] = true;
    }
  }
  static int sm_count[kMaxDevices] = {0};
  if (sm_count[dev] == 0) AEG_CHECK_CUDA(cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
  const int levels = (max_seqlen + 2 * kTM - 1) / (2 * kTM);
  const int64_t items = int64_t(Hq) * B * levels;
  if (items > int64_t(0x7fffffff))
    return set_error(AEG_ERR_INVALID_ARGUMENT, "prefill_attention: %lld work items exceed 2^31", (long long)items);
  static std::atomic<unsigned> launches{0};
  const int slot = static_cast<int>(launches.fetch_add(1) % kCounterSlots);
  const unsigned ctas = static_cast<unsigned>(std::min<int64_t>(sm_count[dev], items));
  prefill_tc_kernel<T><<<ctas, kTThreads, TcLayout::kSmem, stream>>>(
      qm, km, vm, static_cast<T*>(out), o_stride, cu, num_tokens, B, Hq, levels, max_seqlen, Hq / Hkv,
      static_cast<float>(static_cast<double>(scale) * 1.4426950408889634), slot);
  AEG_CHECK_LAUNCH("prefill_attention(tcgen05)");
  return AEG_OK;
}

}  // namespace

uint32_t deverr_read_and_clear_prefill(cudaStream_t s, cudaError_t* err) {
  uint32_t v = 0, zero = 0;
  *err = cudaMemcpyFromSymbolAsync(&v, g_deverr_prefill, sizeof(v), 0, cudaMemcpyDeviceToHost, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  if (*err == cudaSuccess) *err = cudaMemcpyToSymbolAsync(g_deverr_prefill, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
  if (*err == cudaSuccess) *err = cudaStreamSynchronize(s);
  return v;
}

}  // namespace aeg

extern "C" {

int aeg_prefill_attention(void* out, int64_t out_stride, const void* q, int64_t q_stride, const void* k,
                          int64_t k_stride, const void* v, int64_t v_stride, const int32_t* cu_seqlens,
                          int64_t num_tokens, int B, int max_seqlen, int Hq, int Hkv, int D, float scale, int dtype,
                          void* stream) {
  AEG_CHECK_ARG(B >= 0 && max_seqlen >= 0 && num_tokens >= 0, "prefill_attention: negative batch, length or tokens");
  if (B == 0 || max_seqlen == 0 || num_tokens == 0) return AEG_OK;
  AEG_CHECK_ARG(out && q && k && v && cu_seqlens, "prefill_attention: null pointer");
  AEG_CHECK_ARG(Hkv > 0 && Hq > 0 && Hq % Hkv == 0, "prefill_attention: Hq (%d) must be a positive multiple of Hkv (%d)", Hq, Hkv);
  if (D != aeg::kPD) return aeg::set_error(AEG_ERR_UNSUPPORTED, "prefill_attention: head_dim %d not supported (only 128)", D);
  AEG_CHECK_ARG(dtype == AEG_DTYPE_FP16 || dtype == AEG_DTYPE_BF16, "prefill_attention: dtype must be fp16 or bf16");
  AEG_CHECK_ARG(q_stride >= int64_t(Hq) * D && out_stride >= int64_t(Hq) * D && k_stride >= int64_t(Hkv) * D &&
                    v_stride >= int64_t(Hkv) * D,
                "prefill_attention: token strides smaller than heads x head_dim");
  AEG_CHECK_ARG(aeg::aligned(q, 16) && aeg::aligned(k, 16) && aeg::aligned(v, 16) && aeg::aligned(out, 4) &&
                    q_stride % 8 == 0 && k_stride % 8 == 0 && v_stride % 8 == 0 && out_stride % 2 == 0,
                "prefill_attention: q/k/v must be 16-byte aligned with token strides that are multiples of 8 elements");
  AEG_CHECK_ARG(max_seqlen <= 65535 * 256 && B <= 65535 && Hq <= 65535, "prefill_attention: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  AEG_CHECK_ARG(aeg::aligned(out, 16) && out_stride % 8 == 0,
                "prefill_attention: out must be 16-byte aligned with a token stride that is a multiple of 8");
  if (dtype == AEG_DTYPE_BF16)
    return aeg::launch_prefill_tc<__nv_bfloat16>(out, out_stride, q, q_stride, k, k_stride, v, v_stride, cu_seqlens,
                                                 num_tokens, B, max_seqlen, Hq, Hkv, scale, dtype, s);
  return aeg::launch_prefill_tc<__half>(out, out_stride, q, q_stride, k, k_stride, v, v_stride, cu_seqlens, num_tokens,
                                        B, max_seqlen, Hq, Hkv, scale, dtype, s);
}

}  // extern "C"
