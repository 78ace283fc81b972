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
// Kernel: one CTA = 64 query rows of one head of one prompt (4 warps x 16 rows). K and V tiles
// of 64 keys are double-buffered in shared memory with cp.async (16-byte chunks, XOR-swizzled
// rows so that ldmatrix is conflict-free); S = Q K^T and O += P V run on mma.sync m16n8k16 with
// fp32 accumulation, the softmax online in the exp2 domain; P re-enters the MMA as the input
// dtype straight from the S fragments. Tiles are visited heaviest first (the last query tile
// of a prompt sees the most keys).
#include "aeg_common.cuh"

#include <mutex>
#include <type_traits>

namespace aeg {
namespace {

__device__ unsigned int g_deverr_prefill = 0;

constexpr int kPD = 128;        // head dim
constexpr int kPM = 64;         // query rows per CTA
constexpr int kPN = 64;         // keys per tile
constexpr int kPWarps = 4;      // 16 query rows each
constexpr int kPThreads = kPWarps * 32;
constexpr int kRowBytes = kPD * 2;                    // 256 bytes per row
constexpr int kTileBytes = kPN * kRowBytes;           // 16 KiB
constexpr int kPSmem = kPM * kRowBytes + 4 * kTileBytes;  // Q + 2 x (K, V) = 80 KiB

__device__ __forceinline__ float ex2p(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk `c` (0..15) of row `r` in a swizzled 256-byte-row tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * kRowBytes + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // 0 source bytes: the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Rows [row0, row0 + 64) of a [tokens, stride] matrix at column col0 into a swizzled tile;
// rows at or beyond `rows` are zero-filled.
template <typename T>
__device__ __forceinline__ void load_tile(uint32_t tile, const T* base, int64_t stride, int row0, int rows) {
  for (int i = threadIdx.x; i < kPN * 16; i += kPThreads) {
    const int r = i >> 4, c = i & 15;
    const bool valid = row0 + r < rows;
    const T* src = base + static_cast<int64_t>(valid ? row0 + r : 0) * stride + c * 8;
    cp_async16(tile + swz(r, c), src, valid);
  }
}

template <typename T>
__global__ void __launch_bounds__(kPThreads, 2)
prefill_attn_kernel(const T* __restrict__ q, int64_t q_stride, const T* __restrict__ k, int64_t k_stride,
                    const T* __restrict__ v, int64_t v_stride, T* __restrict__ out, int64_t o_stride,
                    const int32_t* __restrict__ cu_seqlens, int64_t num_tokens, int max_seqlen, int G,
                    float scale_log2) {
  using Mma = MmaF32<T>;
  // bf16 P enters O += P V as its bf16 value plus the bf16 rounding residue (two MMAs), ~16
  // mantissa bits, so that bf16 outputs stay within the fp16 path's error; fp16 P as is.
  constexpr bool kSplitP = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(128) uint8_t psmem[];
  const int tile_m = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);  // heaviest first
  const int h = blockIdx.y, b = blockIdx.z;
  const int s0 = cu_seqlens[b];
  const int L = cu_seqlens[b + 1] - s0;
  // a prompt outside the q/k/v rows (or longer than max_seqlen) is skipped and reported
  if (s0 < 0 || L < 0 || static_cast<int64_t>(s0) + L > num_tokens || L > max_seqlen) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && h == 0) atomicOr(&g_deverr_prefill, AEG_DEVERR_SEQ_LEN_RANGE);
    return;
  }
  const int q0 = tile_m * kPM;
  if (L == 0 || q0 >= L) return;
  const int kvh = h / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = lane >> 2, quad = lane & 3;

  const uint32_t sQ = smem_u32(psmem);
  // buffer i: K at kv_buf(i), V right after it
  auto kv_buf = [&](int i) { return sQ + kPM * kRowBytes + static_cast<uint32_t>(i) * 2 * kTileBytes; };

  const T* qb = q + static_cast<int64_t>(s0) * q_stride + static_cast<int64_t>(h) * kPD;
  const T* kb = k + static_cast<int64_t>(s0) * k_stride + static_cast<int64_t>(kvh) * kPD;
  const T* vb = v + static_cast<int64_t>(s0) * v_stride + static_cast<int64_t>(kvh) * kPD;

  const int kv_end = min(L, q0 + kPM);  // causal: the tile's last row sees keys < q0 + 64
  const int n_tiles = (kv_end + kPN - 1) / kPN;

  load_tile(sQ, qb, q_stride, q0, L);
  load_tile(kv_buf(0), kb, k_stride, 0, L);
  load_tile(kv_buf(0) + kTileBytes, vb, v_stride, 0, L);
  cp_async_commit();

  // Q fragments of this warp's 16 rows (A operand), loaded once the first group lands.
  uint32_t qa[8][4];
  float o[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int row_a = q0 + warp * 16 + grp;  // rows of this thread's accumulator entries (within the prompt)
  const int row_b = row_a + 8;

  for (int j = 0; j < n_tiles; ++j) {
    const int cur = j & 1;
    if (j + 1 < n_tiles) {
      load_tile(kv_buf(cur ^ 1), kb, k_stride, (j + 1) * kPN, L);
      load_tile(kv_buf(cur ^ 1) + kTileBytes, vb, v_stride, (j + 1) * kPN, L);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        ldmatrix_x4(qa[ks], sQ + swz(warp * 16 + (lane & 15), ks * 2 + (lane >> 4)));
    }

    const uint32_t sK = kv_buf(cur), sV = sK + kTileBytes;
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // two n-tiles per ldmatrix.x4
        uint32_t kf[4];
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldmatrix_x4(kf, sK + swz(key, ks * 2 + ((lane >> 3) & 1)));
        Mma::run(s[2 * np], qa[ks], kf[0], kf[1]);
        Mma::run(s[2 * np + 1], qa[ks], kf[2], kf[3]);
      }
    }

    // Mask (causal, prompt end), scale into the exp2 domain, online softmax.
    const int key0 = j * kPN;
    const bool need_mask = key0 + kPN - 1 > q0 || key0 + kPN > L;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = key0 + nt * 8 + 2 * quad + e;
        float a = s[nt][e] * scale_log2, c = s[nt][2 + e] * scale_log2;
        if (need_mask) {
          if (key > row_a || key >= L) a = -INFINITY;
          if (key > row_b || key >= L) c = -INFINITY;
        }
        s[nt][e] = a;
        s[nt][2 + e] = c;
        mx0 = fmaxf(mx0, a);
        mx1 = fmaxf(mx1, c);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float base0 = n0 == -INFINITY ? 0.f : n0, base1 = n1 == -INFINITY ? 0.f : n1;
    const float al0 = ex2p(m0 - base0), al1 = ex2p(m1 - base1);  // m = -inf gives 0
    m0 = n0;
    m1 = n1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[4][4];  // P as A fragments of O += P V (k = 16 keys per step)
    uint32_t pr[4][4];  // bf16 only: the rounding residue of P
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = ex2p(s[nt][0] - base0), p1 = ex2p(s[nt][1] - base0);
      const float p2 = ex2p(s[nt][2] - base1), p3 = ex2p(s[nt][3] - base1);
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      const uint32_t h01 = pack2<T>(p0, p1), h23 = pack2<T>(p2, p3);
      pa[nt >> 1][(nt & 1) * 2] = h01;
      pa[nt >> 1][(nt & 1) * 2 + 1] = h23;
      if constexpr (kSplitP) {
        const float2 r01 = unpack2<T>(h01), r23 = unpack2<T>(h23);
        pr[nt >> 1][(nt & 1) * 2] = pack2<T>(p0 - r01.x, p1 - r01.y);
        pr[nt >> 1][(nt & 1) * 2 + 1] = pack2<T>(p2 - r23.x, p3 - r23.y);
      }
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= al0;
      o[nt][1] *= al0;
      o[nt][2] *= al1;
      o[nt][3] *= al1;
    }
    // O += P V: 4 k-steps of 16 keys, 16 n-tiles of 8 dims (two per ldmatrix.x4.trans).
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t vf[4];
        const int m = lane >> 3;
        const int key = kk * 16 + (lane & 7) + ((m & 1) << 3);
        ldmatrix_x4_trans(vf, sV + swz(key, dp * 2 + (m >> 1)));
        Mma::run(o[2 * dp], pa[kk], vf[0], vf[1]);
        Mma::run(o[2 * dp + 1], pa[kk], vf[2], vf[3]);
        if constexpr (kSplitP) {
          Mma::run(o[2 * dp], pr[kk], vf[0], vf[1]);
          Mma::run(o[2 * dp + 1], pr[kk], vf[2], vf[3]);
        }
      }
    }
    __syncthreads();  // the buffer is refilled by the next iteration's loads
  }
  cp_async_wait<0>();

  // Finish: the row sums live spread over the quad.
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  T* ob = out + static_cast<int64_t>(s0) * o_stride + static_cast<int64_t>(h) * kPD;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + 2 * quad;
    if (row_a < L)
      *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(row_a) * o_stride + d) = pack2<T>(o[nt][0] * inv0, o[nt][1] * inv0);
    if (row_b < L)
      *reinterpret_cast<uint32_t*>(ob + static_cast<int64_t>(row_b) * o_stride + d) = pack2<T>(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

template <typename T>
int launch_prefill(void* out, int64_t o_stride, const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                   const void* v, int64_t v_stride, const int32_t* cu, int64_t num_tokens, int B, int max_seqlen,
                   int Hq, int Hkv, float scale, cudaStream_t stream) {
  constexpr int kMaxDevices = 64;
  static bool configured[kMaxDevices] = {false};
  static std::mutex mu;
  int dev = 0;
  AEG_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(AEG_ERR_UNSUPPORTED, "prefill_attention: device %d", dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!configured[dev]) {
      AEG_CHECK_CUDA(cudaFuncSetAttribute(prefill_attn_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem));
      configured[dev] = true;
    }
  }
  const dim3 grid(static_cast<unsigned>((max_seqlen + kPM - 1) / kPM), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  prefill_attn_kernel<T><<<grid, kPThreads, kPSmem, stream>>>(
      static_cast<const T*>(q), q_stride, static_cast<const T*>(k), k_stride, static_cast<const T*>(v), v_stride,
      static_cast<T*>(out), o_stride, cu, num_tokens, max_seqlen, Hq / Hkv, static_cast<float>(static_cast<double>(scale) * 1.4426950408889634));
  AEG_CHECK_LAUNCH("prefill_attention");
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
  AEG_CHECK_ARG(max_seqlen <= (1 << 24) && B <= 65535 && Hq <= 65535, "prefill_attention: grid too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == AEG_DTYPE_BF16)
    return aeg::launch_prefill<__nv_bfloat16>(out, out_stride, q, q_stride, k, k_stride, v, v_stride, cu_seqlens,
                                              num_tokens, B, max_seqlen, Hq, Hkv, scale, s);
  return aeg::launch_prefill<__half>(out, out_stride, q, q_stride, k, k_stride, v, v_stride, cu_seqlens, num_tokens, B,
                                     max_seqlen, Hq, Hkv, scale, s);
}

}  // extern "C"
