/*
 * aegaeon_b200 — C ABI of the B200-native per-token serving path of Aegaeon.
 *
 * The library replaces these operations of the reference serving path:
 *
 *   aeg_swap               aegaeon/ops/swap.cu:25-60 (declared aegaeon/ops/ops.h:4-10,
 *                          bound to Python at aegaeon/ops/ops.cpp:4-5 as `aegaeon.ops.swap`)
 *   aeg_copy_blocks        vLLM 0.5.1 `_C_cache_ops.copy_blocks` (the API that the reference's
 *                          GPU->GPU migration stubs at aegaeon/aegaeon/block_manager.py:876-950
 *                          and aegaeon/aegaeon/worker.py:841-858 would call)
 *   aeg_reshape_and_cache  vLLM 0.5.1 `_C_cache_ops.reshape_and_cache_flash`, reached per layer
 *                          from the model forward at aegaeon/aegaeon/worker.py:517-523
 *   aeg_migrate_blocks     the GPU->GPU migration the reference stubs (worker.py:841-872), with
 *   aeg_ipc_export/open    the KV-cache IPC handle exchange it plans (cuda_wrapper.py:77-104)
 *   aeg_copy_segments      the per-parameter weight-switch copies (worker.py:358-365)
 *   aeg_prefill_attention  vLLM 0.5.1 FlashAttention backend prompt call `flash_attn_varlen_func`
 *   aeg_prepare_step_inputs the per-step Python loops of Worker._prepare_model_inputs
 *                          (worker.py:596-682), on the device
 *   aeg_decode_plan +      vLLM 0.5.1 FlashAttention backend decode call
 *   aeg_paged_attn_decode  `flash_attn_with_kvcache(q, K_l, V_l, block_table, cache_seqlens, ...)`
 *                          with the metadata built at aegaeon/aegaeon/worker.py:554-713
 *
 * Conventions shared by every entry point:
 *   - Pointers are plain addresses; sizes are element or byte counts as named.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Every call is asynchronous on `stream` and returns an aeg_status; 0 is success.
 *     On a non-zero status nothing was enqueued and aeg_last_error() (thread-local)
 *     describes the problem.
 *   - Host-side validation (shapes, alignment, id ranges of host id lists) happens before
 *     any launch. Device-resident ids and slots that are out of range are skipped by the
 *     kernels and reported through the device error word (aeg_read_device_errors).
 *
 * KV-cache geometry (Aegaeon's storage layout, aegaeon/aegaeon/worker.py:388-451 and
 * aegaeon/aegaeon/config.py:256-271): kv_cache[num_blocks][L][2][16][Hkv][D], 16 tokens per
 * block. Per layer l, the K view is kv_cache[:, l, 0] and the V view is kv_cache[:, l, 1]; both
 * have a block stride of L*2*16*Hkv*D elements and a contiguous (16, Hkv, D) block interior.
 * The attention and cache-write entry points take K and V base pointers plus that block
 * stride, so vLLM's own (2, N, 16, Hkv, D) layout works as well.
 */
#ifndef AEGAEON_B200_H_
#define AEGAEON_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AEG_API __attribute__((visibility("default")))
#else
#define AEG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  AEG_OK = 0,
  AEG_ERR_INVALID_ARGUMENT = 1, /* shape, range, alignment or null-pointer problem */
  AEG_ERR_CUDA = 2,             /* a CUDA runtime/driver call failed */
  AEG_ERR_UNSUPPORTED = 3,      /* valid input this build does not handle (e.g. head_dim) */
} aeg_status;

typedef enum {
  AEG_DTYPE_FP16 = 0,
  AEG_DTYPE_BF16 = 1,
} aeg_dtype;

/* Device error bits (aeg_read_device_errors). */
#define AEG_DEVERR_BLOCK_ID_RANGE 0x1u /* a block id outside [0, num_blocks) was skipped   */
#define AEG_DEVERR_SLOT_RANGE 0x2u     /* a cache slot outside [0, num_blocks*16) skipped   */
#define AEG_DEVERR_SEQ_LEN_RANGE 0x4u  /* seq_len < 0 or > 16 * block-table width, clamped  */
#define AEG_DEVERR_WAIT_TIMEOUT 0x8u   /* a bounded pipeline wait gave up (output invalid)   */
#define AEG_DEVERR_PLAN_MISMATCH 0x10u /* the workspace plan does not fit this call; skipped  */

/* Library version (major*10000 + minor*100 + patch). */
AEG_API int aeg_version(void);

/* Message for the last non-zero status returned on the calling thread. */
AEG_API const char* aeg_last_error(void);

/* Reads and clears the sticky device error word of the current device (synchronises
 * `stream`). *flags receives an OR of AEG_DEVERR_* bits raised since the last read. */
AEG_API int aeg_read_device_errors(void* stream, uint32_t* flags);

/* ---------------------------------------------------------------------------------------
 * a1. swap — replaces aegaeon/ops/swap.cu:25-60 (`ops.swap(source_block_ids,
 * target_block_ids, is_swap_in, kv_cache, kv_swap)`).
 *
 * Copies whole blocks of `block_bytes` between the device pool `dev_pool` (n_dev_blocks
 * blocks) and the host pool `host_pool` (n_host_blocks blocks): for i < n,
 *   is_swap_in != 0: dev_pool[dst_ids[i]]  <- host_pool[src_ids[i]]   (H2D)
 *   is_swap_in == 0: host_pool[dst_ids[i]] <- dev_pool[src_ids[i]]    (D2H)
 * `src_ids`/`dst_ids` are HOST arrays (the reference passes std::vector<int64_t>). Every id is
 * range-checked on the host before anything is enqueued (the reference checks nothing).
 * Consecutive ids that are adjacent on both sides are merged into one transfer. The host pool
 * should be page-locked (cudaHostRegister / cudaHostAlloc) for the copy to be asynchronous.
 */
AEG_API int aeg_swap(void* dev_pool, void* host_pool, size_t block_bytes, int64_t n_dev_blocks,
             int64_t n_host_blocks, const int64_t* src_ids, const int64_t* dst_ids, int64_t n,
             int is_swap_in, void* stream);

/* a1 (SM-driven variant). Same data movement as aeg_swap, done by a kernel that reads and
 * writes the page-locked host pool through its mapped device address, so any number of
 * scattered blocks costs one launch. `d_src_ids`/`d_dst_ids` are DEVICE int64 arrays; ids out
 * of range are skipped and raise AEG_DEVERR_BLOCK_ID_RANGE. `host_pool` must be page-locked
 * and mapped (cudaHostGetDevicePointer must succeed for it), else AEG_ERR_INVALID_ARGUMENT. */
AEG_API int aeg_swap_sm(void* dev_pool, void* host_pool, size_t block_bytes, int64_t n_dev_blocks,
                int64_t n_host_blocks, const int64_t* d_src_ids, const int64_t* d_dst_ids,
                int64_t n, int is_swap_in, void* stream);

/* ---------------------------------------------------------------------------------------
 * a8. copy_blocks — the vLLM 0.5.1 `copy_blocks` operation on Aegaeon's whole-block layout.
 * For i < n: pool[dst_ids[i]] <- pool[src_ids[i]] (block_bytes each). `d_src_ids`/`d_dst_ids`
 * are DEVICE int64 arrays. Pairs are applied concurrently: a block that is both a source and a
 * destination within one call gives an unspecified result (as in vLLM). Out-of-range ids are
 * skipped and raise AEG_DEVERR_BLOCK_ID_RANGE.
 */
AEG_API int aeg_copy_blocks(void* pool, size_t block_bytes, int64_t num_blocks, const int64_t* d_src_ids,
                    const int64_t* d_dst_ids, int64_t n, void* stream);

/* ---------------------------------------------------------------------------------------
 * f1. GPU <-> GPU KV block migration over NVLink. Replaces the reference's stubbed migration
 * path: Worker.register_kvcache_mem_handles / Worker.migrate_blocks
 * (aegaeon/aegaeon/worker.py:841-872) and BlockManager._migrate_requests
 * (aegaeon/aegaeon/block_manager.py:876-950), which hand the target engine the source
 * engine's KV-cache CUDA IPC handles (aegaeon/aegaeon/cuda_wrapper.py:77-104, 190-208:
 * cudaIpcGetMemHandle / cudaIpcOpenMemHandle with lazy peer access) so that the target pulls
 * a request's blocks into blocks of its own pool.
 *
 * An AEG_IPC_HANDLE_BYTES-byte handle names a device pool of the exporting process: the CUDA
 * IPC handle of the allocation that holds it, the pool's offset in that allocation and the
 * allocation's size (so the importer can range-check). Handles are plain bytes: send them
 * through any host channel (a torch.distributed store, a pipe).
 */
#define AEG_IPC_HANDLE_BYTES 96

/* Fills `handle_out` (AEG_IPC_HANDLE_BYTES bytes) for the device pool at `dev_pool`, which
 * must lie in memory from cudaMalloc (e.g. a tensor of PyTorch's default allocator). */
AEG_API int aeg_ipc_export(const void* dev_pool, void* handle_out);

/* Maps the pool named by `handle` (exported by another process) into this process and stores
 * its address in *dev_pool_out; *pool_bytes_out (may be NULL) receives the bytes from that
 * address to the end of the exporter's allocation. Opening a handle that this process has
 * already opened returns the same mapping (reference counted). */
AEG_API int aeg_ipc_open(const void* handle, void** dev_pool_out, int64_t* pool_bytes_out);

/* Releases a mapping returned by aeg_ipc_open (after work that reads it has completed). */
AEG_API int aeg_ipc_close(void* dev_pool);

/* For i < n: dst_pool[d_dst_ids[i]] <- src_pool[d_src_ids[i]] (block_bytes each), by a kernel
 * on the current device. One pool is normally this GPU's and the other a peer GPU's (mapped by
 * aeg_ipc_open, or a peer allocation of this process): the kernel pulls (peer source) or pushes
 * (peer target) 16-byte vectors over NVLink. Before any launch the host checks that both pools
 * are device memory that the current device can address (peer access is enabled when needed)
 * and that [pool, pool + num_blocks * block_bytes) lies inside each pool's allocation.
 * `d_src_ids`/`d_dst_ids` are DEVICE int64 arrays on the current device; ids out of range are
 * skipped and raise AEG_DEVERR_BLOCK_ID_RANGE. Target blocks must be distinct. */
AEG_API int aeg_migrate_blocks(void* dst_pool, int64_t n_dst_blocks, const void* src_pool,
                               int64_t n_src_blocks, size_t block_bytes, const int64_t* d_src_ids,
                               const int64_t* d_dst_ids, int64_t n, void* stream);

/* Copy-engine form of aeg_migrate_blocks: HOST id arrays, every id range-checked before anything
 * is enqueued, one cudaMemcpyAsync per run of blocks adjacent on both sides. */
AEG_API int aeg_migrate_blocks_dma(void* dst_pool, int64_t n_dst_blocks, const void* src_pool,
                                   int64_t n_src_blocks, size_t block_bytes, const int64_t* src_ids,
                                   const int64_t* dst_ids, int64_t n, void* stream);

/* ---------------------------------------------------------------------------------------
 * f4. Per-step model inputs on the device. Replaces the Python loops of
 * Worker._prepare_model_inputs (aegaeon/aegaeon/worker.py:596-682; padding utils.py:241-257)
 * for a batch whose block tables stay resident on the device between steps.
 *
 * Inputs (DEVICE): block_tables int32 [B, table_stride], row i holding request i's blocks in
 * order; context_lens, seq_lens int32 [B] (tokens already cached / after this step).
 * Outputs (DEVICE), for the T = sum(seq_len - context_len) new tokens in request order:
 *   slot_mapping, positions  int64 [capacity]: position p of request i and its slot
 *                            block_tables[i][p / 16] * 16 + p % 16 (worker.py:612-633)
 *   query_lens               int64 [B]      seq_len - context_len
 *   query_start_loc          int32 [B + 1]  exclusive cumulative sums of query_lens / seq_lens
 *   seq_start_loc            int32 [B + 1]  (worker.py:653-676)
 *   attn_tables (or NULL)    int32 [B, table_stride]: the rows attention reads, as the reference
 *                            builds them (worker.py:603-609, 640-646): a decode request's
 *                            ceil(seq_len / 16) blocks then zeros, a prompt's row all zeros
 *   num_tokens               int64 [1]      T
 * A request with context_len < 0, seq_len < context_len or seq_len > 16 * table_stride gets no new
 * tokens and raises AEG_DEVERR_SEQ_LEN_RANGE; when T > capacity the tokens past capacity are not
 * written and AEG_DEVERR_SLOT_RANGE is raised (num_tokens still holds T). Two launches. */
AEG_API int aeg_prepare_step_inputs(const int32_t* block_tables, int table_stride,
                                    const int32_t* context_lens, const int32_t* seq_lens, int B,
                                    int64_t* slot_mapping, int64_t* positions, int64_t capacity,
                                    int64_t* query_lens, int32_t* query_start_loc,
                                    int32_t* seq_start_loc, int32_t* attn_tables,
                                    int64_t* num_tokens, void* stream);

/* Applies n updates to the DEVICE tables [rows, table_stride]: d_updates is a DEVICE int32 array
 * of (row, column, block id) triples (the blocks a step appended or a new request's row).
 * Triples outside the table are skipped and raise AEG_DEVERR_BLOCK_ID_RANGE. Updates to one
 * cell within a call land in an unspecified order. */
AEG_API int aeg_update_block_tables(int32_t* block_tables, int table_stride, int rows,
                                    const int32_t* d_updates, int64_t n, void* stream);

/* ---------------------------------------------------------------------------------------
 * f3. Model-weight switch: the prefetched model's parameters, page-locked host model cache ->
 * device weight arena, in one call. Replaces the per-parameter loop of the reference
 * (`new_storage.copy_(param.untyped_storage(), non_blocking=True)` for every parameter,
 * aegaeon/aegaeon/worker.py:358-365; model cache registered at aegaeon/aegaeon/loader/loader.py:187-197;
 * device slices from the bump allocator, aegaeon/aegaeon/allocator.py:54-81).
 *
 * For i < n: copies sizes[i] bytes from src_base + src_offsets[i] to dst_base + dst_offsets[i]
 * (HOST arrays, all validated before anything is enqueued; destination segments must not
 * overlap). engine:
 *   AEG_COPY_ENGINE_DMA  one cudaMemcpyAsync per run of segments adjacent on both sides;
 *                        `workspace` unused.
 *   AEG_COPY_ENGINE_SM   one kernel for all segments through the mapped address of page-locked
 *                        host memory (device memory as is); needs a device `workspace` of
 *                        aeg_copy_segments_workspace_size(n) bytes, into which the segment table is
 *                        staged with a pageable copy (that copy first waits for earlier work on
 *                        `stream`). */
#define AEG_COPY_ENGINE_DMA 0
#define AEG_COPY_ENGINE_SM 1
AEG_API size_t aeg_copy_segments_workspace_size(int64_t n);
AEG_API int aeg_copy_segments(void* dst_base, const void* src_base, const int64_t* src_offsets,
                              const int64_t* dst_offsets, const int64_t* sizes, int64_t n, int engine,
                              void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------
 * f2. Prefill (prompt) attention. Replaces vLLM 0.5.1's FlashAttention backend call for prompts,
 * `flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
 * softmax_scale, causal=True)` with q and k lengths equal (Aegaeon prefills whole prompts without
 * chunking, aegaeon/aegaeon/worker.py:603-626; the prompt's K/V also go to the paged cache
 * through aeg_reshape_and_cache).
 *
 * q [num_tokens, Hq, D], k/v [num_tokens, Hkv, D], out [num_tokens, Hq, D] (token strides in
 * elements; q/k/v 16-byte aligned with strides that are multiples of 8), prompt b = tokens
 * cu_seqlens[b] .. cu_seqlens[b + 1] - 1 (DEVICE int32 [B + 1]); max_seqlen >= every prompt's
 * length. For query token i of a prompt:
 *   out[i, h] = softmax_j(scale * q[i, h] . k[j, h / (Hq / Hkv)]) . v[j, h / (Hq / Hkv)], j = 0 .. i
 * fp32 accumulation, output rounded to the input dtype. D = 128. A prompt whose range leaves
 * [0, num_tokens) or exceeds max_seqlen is skipped (its rows are not written) and raises
 * AEG_DEVERR_SEQ_LEN_RANGE. The launch is persistent (one CTA per SM) and takes its work from a
 * device counter, one of 64 the library rotates over per launch (each launch's last CTA resets
 * its own): launches on several streams may overlap as long as fewer than 64 are in flight at
 * once; a CUDA graph that holds a launch reuses that launch's counter at every replay, so two
 * replays of one graph are not run concurrently. */
AEG_API int aeg_prefill_attention(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                                  const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                                  const int32_t* cu_seqlens, int64_t num_tokens, int B, int max_seqlen,
                                  int Hq, int Hkv, int D, float scale, int dtype, void* stream);

/* ---------------------------------------------------------------------------------------
 * a6. reshape_and_cache — replaces vLLM 0.5.1 `reshape_and_cache_flash(key, value, key_cache,
 * value_cache, slot_mapping, "auto")` as called per layer inside the model forward
 * (aegaeon/aegaeon/worker.py:517-523, slot mapping built at worker.py:628-633).
 *
 * For t < T with s = slot_mapping[t] >= 0:
 *   k_cache[(s / 16) * block_stride + (s % 16) * Hkv * D + h * D + d] = key[t * key_stride + h * D + d]
 * and the same for value/v_cache. Slots < 0 are skipped (padding), as in vLLM. Slots
 * >= num_blocks * 16 are skipped and raise AEG_DEVERR_SLOT_RANGE. Elements are 2 bytes
 * (fp16 or bf16; the copy is bit-exact and dtype-blind). `key_stride`/`value_stride` are the
 * token strides of key/value in elements; `block_stride` is in elements.
 */
AEG_API int aeg_reshape_and_cache(const void* key, const void* value, int64_t key_stride,
                          int64_t value_stride, void* k_cache, void* v_cache,
                          int64_t block_stride, int64_t num_blocks,
                          const int64_t* slot_mapping, int64_t T, int Hkv, int D, void* stream);

/* ---------------------------------------------------------------------------------------
 * a7. Paged decode attention — replaces the decode half of the vLLM 0.5.1 FlashAttention
 * backend: flash_attn_with_kvcache(q[:, None], K_l, V_l, block_table=block_tables,
 * cache_seqlens=seq_lens, softmax_scale=scale, causal=True) with one query token per
 * sequence. For b < B, h < Hq, with G = Hq / Hkv and n = seq_lens[b]:
 *   out[b, h] = sum_{j<n} softmax_j(scale * q[b,h] . K[blk(b,j), j%16, h/G]) * V[blk(b,j), j%16, h/G]
 *   blk(b, j) = block_tables[b * table_stride + j / 16]
 * computed in fp32 and rounded to the storage dtype. seq_len 0 gives a zero row.
 *
 * A decode step runs aeg_decode_plan once (it depends only on seq_lens and block_tables, like
 * the per-step attention metadata at worker.py:694-711) and then aeg_paged_attn_decode (or
 * aeg_decode_layer) once per layer with the same workspace. The workspace is caller-owned device
 * memory of at least aeg_decode_workspace_size(B, Hq, Hkv, D) bytes, 256-byte aligned, used by
 * one stream at a time. The plan cuts the batch's (block, KV head) items, in
 * (sequence, head) order, into one contiguous range of equal cost per worker warp of the
 * attention grid (8 warps x one CTA per SM); a (sequence, head) cut across warps is merged at
 * the end of the same launch, each merge waiting only for the warps that computed its pieces.
 *
 * Supported: D = 128; Hq % Hkv == 0; Hq / Hkv <= 16; fp16 or bf16; 16-byte aligned K/V
 * bases; a block stride that is a multiple of 8 elements; q/out with even token strides.
 */
AEG_API size_t aeg_decode_workspace_size(int B, int Hq, int Hkv, int D);

AEG_API int aeg_decode_plan(void* workspace, size_t workspace_bytes, const int32_t* block_tables,
                            int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv, int D,
                            void* stream);

/* Flags of aeg_paged_attn_decode / aeg_decode_layer. AEG_DECODE_PREFETCH: the K/V cache blocks
 * and block tables the call reads are not written by the kernel that immediately precedes it on
 * `stream`, so the launch may request its first K/V tiles before that kernel has finished (the
 * query rows and new K/V rows are still read only after it). Safe between consecutive layers of
 * one decode step (a layer writes only its own layer's rows); not after a cache write, a block
 * copy or a swap of the same layer.
 * AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE (aeg_paged_attn_decode): the kernel that immediately
 * precedes the call wrote, of what the call reads, at most position seq_lens[b] - 1 of each
 * sequence (the decode cache write of aeg_reshape_and_cache with the slots the reference builds
 * for a decode step) and no block table. The launch requests its first tiles early and reads
 * each sequence's newest row again after that kernel has finished. */
#define AEG_DECODE_PREFETCH 0x1
#define AEG_DECODE_PREFETCH_AFTER_DECODE_WRITE 0x2

AEG_API int aeg_paged_attn_decode(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                          const void* k_cache, const void* v_cache, int64_t block_stride,
                          int64_t num_blocks, const int32_t* block_tables, int table_stride,
                          const int32_t* seq_lens, int B, int Hq, int Hkv, int D, float scale,
                          int dtype, void* workspace, size_t workspace_bytes, int flags,
                          void* stream);

/* a6 + a7 fused. One decode layer as the reference runs it per layer (cache write of the new
 * token, then decode attention; aegaeon/aegaeon/worker.py:517-523): for every sequence b with
 * n = seq_lens[b] > 0, the new token's key/value rows (key_new[b], value_new[b], [Hkv, D] each,
 * token strides key_stride/value_stride) are written into position n - 1 of the sequence, i.e.
 * slot block_tables[b][(n-1)/16] * 16 + (n-1) % 16 -- the slot the reference builds for a decode
 * request (worker.py:628-633 with context_len = seq_len - 1) -- and attention then runs over
 * positions [0, n) exactly as aeg_paged_attn_decode, in the same launch. The result equals
 * aeg_reshape_and_cache with those slots followed by aeg_paged_attn_decode.
 * key_new/value_new must be 4-byte aligned with even token strides. */
AEG_API int aeg_decode_layer(void* out, int64_t out_stride, const void* q, int64_t q_stride,
                             const void* key_new, int64_t key_stride, const void* value_new,
                             int64_t value_stride, void* k_cache, void* v_cache,
                             int64_t block_stride, int64_t num_blocks, const int32_t* block_tables,
                             int table_stride, const int32_t* seq_lens, int B, int Hq, int Hkv,
                             int D, float scale, int dtype, void* workspace,
                             size_t workspace_bytes, int flags, void* stream);

/* Allocation-free decode attention. No counterpart in the reference: Aegaeon always has torch's
 * allocator at hand. This entry serves callers that cannot pass a workspace and must not have the
 * library allocate one -- hosts binding only this C ABI with no device allocator of their own,
 * code running inside an allocator or memory-pool callback, serving loops whose device memory is
 * all given to the KV-block pool. It computes what aeg_decode_plan + aeg_paged_attn_decode compute
 * (same arguments minus the workspace) in a fixed 32 MiB scratch area per device that lives in the
 * library's static device memory; nothing is allocated by the call.
 *   - Limit: the scratch holds partial rows for 2 x the device's worker warps (about 8.6 MB at
 *     Hq/Hkv = 7, 20 MB at 16, on a 148-SM B200) plus 48 bytes per (sequence, KV head) pair; a
 *     call needing more than 32 MiB (over ~500K pairs at Hq/Hkv = 7, ~280K at 16) fails with
 *     AEG_ERR_INVALID_ARGUMENT, nothing enqueued.
 *   - Every check (arguments, alignment, tensor maps) runs before the first launch: a call that
 *     returns an error has enqueued nothing and left the scratch as the previous call left it.
 *   - Nothing has to be zeroed by the caller: every call re-plans and resets the flags it uses.
 *   - The scratch is shared by all calls on a device: calls that overlap in time (e.g. on two
 *     unordered streams) race. Keep them on one stream or order them.
 *   - The first call on a device looks up the scratch address and configures the kernel with that
 *     device current; make it before any stream capture begins. */
AEG_API int aeg_paged_attn_decode_noalloc(void* out, int64_t out_stride, const void* q,
                                          int64_t q_stride, const void* k_cache, const void* v_cache,
                                          int64_t block_stride, int64_t num_blocks,
                                          const int32_t* block_tables, int table_stride,
                                          const int32_t* seq_lens, int B, int Hq, int Hkv, int D,
                                          float scale, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AEGAEON_B200_H_ */
