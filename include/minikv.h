/*
 * minikv -- C ABI of the B200 (sm_100a) paged-KV-cache hot path.
 *
 * Drop-in native layer for the reference engine's operator API in
 * mini_engine/kernels (paths below are inside the reference project).  Every
 * entry point takes raw device pointers, element counts and a cudaStream_t
 * passed as void*; nothing here knows about torch.  All launches go on the
 * given stream, never synchronise (except minikv_device_status) and allocate
 * nothing, so they can be captured in a CUDA graph.
 *
 * Layouts (row-major, contiguous unless a stride argument says otherwise):
 *   key/value cache : [num_blocks, block_size, kv_heads, head_dim]  -- one layer
 *                     of the pool [layers, num_blocks, block_size, kv_heads, head_dim]
 *                     (mini_engine/cache/kv_cache.py:50-52)
 *   query / out     : [batch, q_heads, head_dim]        (decode)
 *                     [tokens, q_heads, head_dim]       (prefill)
 *   block_tables    : [rows, table_width] int64, -1 padded
 * dtype codes: MINIKV_F32, MINIKV_F16, MINIKV_BF16 (all tensors of a call share it).
 * head_dim must be one of 16, 32, 64, 80, 96, 128, 192, 256.
 *
 * Return value: MINIKV_OK or an error code; minikv_last_error() then holds a
 * message (thread-local).  Pointers must be 16-byte aligned.
 */
#ifndef MINIKV_H
#define MINIKV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MINIKV_ABI_VERSION 1

enum { MINIKV_F32 = 0, MINIKV_F16 = 1, MINIKV_BF16 = 2 };
/* FP8 KV pool byte formats (OCP FP8). */
enum { MINIKV_FP8_E4M3 = 0, MINIKV_FP8_E5M2 = 1 };
enum { MINIKV_OK = 0, MINIKV_EINVAL = 1, MINIKV_ECUDA = 2, MINIKV_EUNSUPPORTED = 3 };
/* bits of the device status word (minikv_device_status) */
enum { MINIKV_STATUS_WAIT_TIMEOUT = 1 };

int minikv_abi_version(void);

/* SHA-256 (hex) of the sources the library was built from (csrc/*.cu, *.cuh and
 * this header), so a loader can refuse a library older than its sources.  New;
 * the reference JIT-builds its extension on import and has no such check. */
const char* minikv_source_hash(void);

/* Message of the last failed call on this thread ("" if none). */
const char* minikv_last_error(void);

/* Synchronise `stream`, then read (and if clear != 0 reset) the device status
 * word of the current device: kernels set bits there instead of trapping when
 * a bounded wait gives up.  New; the reference has no device status. */
int minikv_device_status(unsigned int* status, int clear, void* stream);

/* Synchronise `stream`, then set the limit (nanoseconds, default 2e9) of the
 * waits in which a kernel's producer waits for its consumers to free a ring
 * slot, on the current device.  When such a wait gives up, the kernel sets
 * MINIKV_STATUS_WAIT_TIMEOUT, issues no more copies, waits for the copies it
 * has issued and runs to its end (outputs of that call are undefined).  A short
 * limit lets a test drive that path without a hang or a fault; production
 * callers leave the default.  New; the reference's kernels have no bounded waits. */
int minikv_set_wait_limit(uint64_t limit_ns, void* stream);

/* ---------------------------------------------------------------- decode ---
 * Split-KV decode attention over paged K/V (GQA: q head h reads kv head
 * h / (q_heads / kv_heads)).  out[b, h] = softmax(q[b,h] . K^T / sqrt(D)) V over
 * the first context_lens[b] tokens of request b's pages.
 * Replaces paged_attention_cuda (mini_engine/kernels/csrc/paged_attention.cu:266-280)
 * behind paged_attention (mini_engine/kernels/paged.py:8-22,
 * mini_engine/kernels/csrc/bindings.cpp:152-184).
 * Trusted-mode guards as in the reference kernel: a page id outside
 * [0, num_blocks) masks its tokens, a length outside [1, table_width*block_size]
 * or a fully masked row gives an all-zero output row.
 * The number of KV splits depends only on (batch, table_width, block_size,
 * heads, head_dim, dtype) and the device, never on context_lens, so a
 * captured graph stays valid when lengths change.
 * workspace: device scratch of at least minikv_paged_decode_workspace_bytes()
 * bytes, zero-filled before its first use (e.g. one cudaMemset) and then
 * reused as is: every call leaves the ticket counters it keeps there at zero.
 * Calls that share a workspace must not overlap on the GPU. */
int64_t minikv_paged_decode_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                            int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                            int64_t table_width, int dtype);
int minikv_paged_decode(const void* query, const void* key_cache, const void* value_cache,
                        const int64_t* block_tables, const int64_t* context_lens, void* out,
                        void* workspace, int64_t workspace_bytes,
                        int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                        int64_t num_blocks, int64_t block_size, int64_t table_width,
                        int dtype, void* stream);

/* minikv_paged_decode for a launch chain: the same arguments and results,
 * for a caller whose context_lens and block_tables were written before the
 * previous kernel on the stream started (typically that kernel is the KV
 * append of the same step, as in NativeQwen3.forward_decode_batch,
 * native_qwen3.py:185-195).  The kernel is launched with programmatic
 * dependent launch and reads the lengths and page tables while the previous
 * kernel finishes; it reads KV, q and the workspace only after that kernel has
 * completed.  Every libminikv kernel is a chained launch that lets its
 * successor start early, so calling this right after minikv_kv_append_batch
 * or minikv_qk_rope_append overlaps the decode prologue with the append.
 * No counterpart in the reference (its decode is launched after a full
 * stream serialisation, bindings.cpp:152-184). */
int minikv_paged_decode_chained(const void* query, const void* key_cache, const void* value_cache,
                                const int64_t* block_tables, const int64_t* context_lens, void* out,
                                void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                                int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                int64_t table_width, int dtype, void* stream);

/* KV append and decode attention in one launch: the result of
 * minikv_kv_append_batch(key/value at token_offsets) followed by
 * minikv_paged_decode over context_lens = token_offsets + 1, with the same
 * guards.  key/value: [batch, kv_heads, head_dim], contiguous.  The new row of
 * request b is written to its pool slot (bit-exact, skipped when the offset
 * is negative, beyond the table or on an invalid page) by the CTA that
 * attends it, which reads it from key/value instead of the pool.  16-bit and
 * fp32 pools; workspace as for minikv_paged_decode (same size).  chained != 0:
 * token_offsets, block_tables and the pool rows the call reads (all but the
 * appended ones) were written before the previous kernel on the stream
 * started; key/value may come from that kernel.  The launch then overlaps the
 * previous kernel's tail: it resolves its pages and starts staging pool rows
 * before waiting for that kernel.  Replaces the two launches of
 * Attention.forward_decode_batch (mini_engine/model/native_qwen3.py:188-196:
 * write_kv_cache_batch, then paged_attention over positions + 1). */
int minikv_paged_decode_append(const void* query, const void* key_cache, const void* value_cache,
                               const int64_t* block_tables, const int64_t* token_offsets, const void* key,
                               const void* value, void* out, void* workspace, int64_t workspace_bytes,
                               int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                               int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype, int chained,
                               void* stream);

/* Same decode attention, for callers that cannot allocate device memory when
 * they call (a CUDA graph being captured under a framework that owns every
 * allocation, a serving loop that bans cudaMalloc after start-up, a cgo/JNI
 * host without a device allocator).  No counterpart in the reference: its
 * kernel always allocates its partials with at::empty.  The scratch lives in a
 * built-in 16 MiB device array that every GPU loading the library keeps until
 * exit; shapes needing more scratch than that fail with MINIKV_EINVAL.  The
 * first call on each device looks the array up (cudaGetSymbolAddress) and
 * should come before any stream capture; the address it keeps is valid for
 * the life of the device's primary context (not across cudaDeviceReset).
 * All calls share the array: calls
 * that overlap on the GPU race and must be serialised by the caller.  Nothing
 * is allocated or freed. */
int minikv_paged_decode_noalloc(const void* query, const void* key_cache, const void* value_cache,
                                const int64_t* block_tables, const int64_t* context_lens, void* out,
                                int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                int64_t num_blocks, int64_t block_size, int64_t table_width,
                                int dtype, void* stream);

/* ------------------------------------------------------------- KV writes ---
 * Bit-exact row copies with 16-byte vector loads/stores.  A source row is the
 * [kv_heads, head_dim] block of one token; consecutive source tokens are
 * `*_token_stride` elements apart (>= kv_heads*head_dim).
 *
 * Scatter rows[slot_mapping[t]] = key[t] (and value), rows = cache viewed as
 * [num_blocks*block_size, kv_heads, head_dim].  Slots outside the capacity are
 * skipped.  Replaces write_kv_cache_slots_cuda
 * (mini_engine/kernels/csrc/data.cu:209-250; data.py:84-130). */
int minikv_kv_scatter_slots(void* key_cache, void* value_cache, const int64_t* slot_mapping,
                            const void* key, const void* value, int64_t tokens,
                            int64_t num_blocks, int64_t block_size, int64_t kv_heads, int64_t head_dim,
                            int64_t key_token_stride, int64_t value_token_stride,
                            int dtype, void* stream);

/* ------------------------------------------------------------ FP8 KV pool ---
 * No counterpart in the reference, which lists an FP8 KV pool as future work
 * (VALIDATION_AND_BENCHMARKS.md:375).  The pool has the 16-bit pool's shape,
 * [num_blocks, block_size, kv_heads, head_dim], one OCP FP8 byte per element,
 * fp8_format MINIKV_FP8_E4M3 (largest finite 448, no infinities) or
 * MINIKV_FP8_E5M2 (largest finite 57344), with one fp32 scale for keys and one
 * for values: stored = fp8(x * (1/scale)), the product rounded to fp32, then
 * to the nearest-even code, saturated to the largest finite value (NaN stays
 * NaN); read as stored * scale.  E5M2 decodes with byte moves only (an E5M2
 * byte is the high byte of an fp16), E4M3 keeps one more mantissa bit.
 *
 * Quantising slot scatter: as minikv_kv_scatter_slots (slots outside the
 * capacity are skipped), from fp32/fp16/bf16 rows (`dtype`) into the byte
 * pools.  kv_heads*head_dim must be a multiple of 16. */
int minikv_kv_scatter_slots_fp8(void* key_cache, void* value_cache, const int64_t* slot_mapping,
                                const void* key, const void* value, int64_t tokens,
                                int64_t num_blocks, int64_t block_size, int64_t kv_heads, int64_t head_dim,
                                int64_t key_token_stride, int64_t value_token_stride,
                                float k_scale, float v_scale, int fp8_format, int dtype, void* stream);

/* Decode attention over an FP8 pool: minikv_paged_decode's contract and
 * guards, with an fp16/bf16 query and output (`dtype`) and K/V read as
 * code * scale.  The products run on fp16 tensor cores: Q is rounded to fp16
 * (saturated at +-65504).  head_dim in {32, 64, 96, 128, 192, 256}.  The
 * workspace (zero-filled before its first use, left zero by every call) has
 * its own size query. */
int64_t minikv_paged_decode_fp8_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                                int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                                int64_t table_width, int dtype);
int minikv_paged_decode_fp8(const void* query, const void* key_cache, const void* value_cache,
                            const int64_t* block_tables, const int64_t* context_lens, void* out,
                            void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                            int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                            int64_t table_width, float k_scale, float v_scale, int fp8_format, int dtype,
                            void* stream);

/* KV append and fp8 decode in one launch: minikv_kv_scatter_slots_fp8 of
 * key/value ([batch, kv_heads, head_dim] in the query dtype, contiguous) at
 * each request's slot for position token_offsets[b], followed by
 * minikv_paged_decode_fp8 over token_offsets + 1.  The new row is quantised
 * into its pool slot (bit-exact with the scatter: fp8(x * (1/scale))) by the
 * CTA that attends it, then staged from the pool; the guards are those of
 * minikv_paged_decode_append.  chained as for minikv_paged_decode_append.  No
 * counterpart in the reference (it has no fp8 pool). */
int minikv_paged_decode_fp8_append(const void* query, const void* key_cache, const void* value_cache,
                                   const int64_t* block_tables, const int64_t* token_offsets, const void* key,
                                   const void* value, void* out, void* workspace, int64_t workspace_bytes,
                                   int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                   int64_t num_blocks, int64_t block_size, int64_t table_width, float k_scale,
                                   float v_scale, int fp8_format, int dtype, int chained, void* stream);

/* Ragged causal paged prefill over an FP8 pool: minikv_paged_prefill's
 * contract (arguments, guards, packed [tokens, q_heads, head_dim] query and
 * output) with fp16/bf16 query/output (`dtype`), K/V read as code * scale.
 * Routes: head_dim 128 on the tensor-core prefill's shapes stages the codes
 * with TMA and converts them to fp16 inside the kernel (fp16 MMAs; no
 * workspace); the other tensor-core shapes run it on a dense copy (in
 * `dtype`) of the table-referenced pages, made in the workspace by a
 * conversion kernel launched first; other shapes, and batches whose copy
 * would pass 8 GiB, run the CUDA-core route (one decode row per query token,
 * fp8 consumer).  The workspace has its own size query (0 bytes: none is
 * read; no zero fill needed). */
int64_t minikv_paged_prefill_fp8_workspace_bytes(int64_t tokens, int64_t requests, int64_t q_heads,
                                                 int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                                                 int64_t block_size, int64_t table_width, int64_t max_query_len,
                                                 int dtype);
int minikv_paged_prefill_fp8(const void* q, const void* key_cache, const void* value_cache,
                             const int64_t* cu_seqlens_q, const int64_t* query_starts, const int64_t* block_tables,
                             const int64_t* context_lens, void* out, void* workspace, int64_t workspace_bytes,
                             int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                             int64_t num_blocks, int64_t block_size, int64_t table_width, int64_t max_query_len,
                             float k_scale, float v_scale, int fp8_format, int dtype, void* stream);

/* Decode append: request r writes its token at logical position
 * token_offsets[r] through block_tables[r]; rows whose page index or physical
 * page is out of range are skipped.  Replaces write_kv_cache_batch_cuda
 * (mini_engine/kernels/csrc/data.cu:175-192; data.py:67-81). */
int minikv_kv_append_batch(void* key_cache, void* value_cache, const int64_t* block_tables,
                           const int64_t* token_offsets, const void* key, const void* value,
                           int64_t batch, int64_t table_width, int64_t num_blocks, int64_t block_size,
                           int64_t kv_heads, int64_t head_dim,
                           int64_t key_token_stride, int64_t value_token_stride,
                           int dtype, void* stream);

/* Contiguous token range [token_offset, token_offset+tokens) through one list
 * of block ids.  Replaces write_kv_cache_cuda
 * (mini_engine/kernels/csrc/data.cu:165-173; data.py:39-64; kv_cache.py:123-145). */
int minikv_kv_write_range(void* key_cache, void* value_cache, const int64_t* block_ids, int64_t num_ids,
                          int64_t token_offset, const void* key, const void* value, int64_t tokens,
                          int64_t num_blocks, int64_t block_size, int64_t kv_heads, int64_t head_dim,
                          int64_t key_token_stride, int64_t value_token_stride,
                          int dtype, void* stream);

/* Copy-on-write: for every (src, dst) pair in `pairs` ([num_pairs, 2] int64,
 * device memory) copy page src to page dst in every layer of both pools
 * ([num_layers, num_blocks, block_elems] with block_elems =
 * block_size*kv_heads*head_dim).  Pairs must have distinct dst pages and no
 * dst may be another pair's src.  The reference has no copy-on-write; this is
 * the kernel behind the new BlockManager fork (block_manager.py:99-116 keeps
 * the refcounts it relies on). */
int minikv_copy_blocks(void* key_pool, void* value_pool, const int64_t* pairs, int64_t num_pairs,
                       int64_t num_layers, int64_t num_blocks, int64_t block_elems,
                       int dtype, void* stream);

/* --------------------------------------------------------------- prefill ---
 * Ragged causal prefill over paged K/V: packed query token t of request r
 * (cu_seqlens_q[r] <= t < cu_seqlens_q[r+1]) sits at position
 * p = query_starts[r] + t - cu_seqlens_q[r] and attends keys [0, p] of r's
 * pages (history and the current chunk, already scattered).
 * Replaces paged_prefill_attention_cuda (mini_engine/kernels/csrc/prefill.cu:200-240;
 * prefill.py:61-131).  bf16/fp16 with head_dim 64 or 128 and a GQA group that
 * divides 128 run on tcgen05 tensor cores (TMEM accumulators, TMA-fed tiles);
 * other shapes run a CUDA-core route.  max_query_len bounds every request's
 * query count (it sizes the grid).  Tokens whose metadata is out of range get
 * zero rows.  workspace: at least minikv_paged_prefill_workspace_bytes(). */
int64_t minikv_paged_prefill_workspace_bytes(int64_t tokens, int64_t requests, int64_t q_heads,
                                             int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                                             int64_t block_size, int64_t table_width,
                                             int64_t max_query_len, int dtype);
int minikv_paged_prefill(const void* q, const void* key_cache, const void* value_cache,
                         const int64_t* cu_seqlens_q, const int64_t* query_starts,
                         const int64_t* block_tables, const int64_t* context_lens, void* out,
                         void* workspace, int64_t workspace_bytes,
                         int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                         int64_t head_dim, int64_t num_blocks, int64_t block_size,
                         int64_t table_width, int64_t max_query_len, int dtype, void* stream);

/* -------------------------------------------------------------- metadata ---
 * Device-side construction of the ragged prefill batch metadata of
 * PrefillBatch.from_sequences (mini_engine/engine/batch.py:67-137) from compact
 * per-request inputs: query_starts[B], cu_seqlens_q[B+1], cu_blocks[B+1] and
 * the concatenated block ids of every request.  Outputs (int64, device):
 * input_ids[T] (copied from token_ids), positions[T], slot_mapping[T],
 * out_cu_seqlens_q[B+1], out_query_starts[B], context_lens[B],
 * block_tables[B, table_width] (-1 padded).  Host code validates first
 * (shared-page writes, duplicates, ranges); the kernel itself only guards
 * its own indices. */
int minikv_build_prefill_metadata(const int64_t* query_starts, const int64_t* cu_seqlens_q,
                                  const int64_t* cu_blocks, const int64_t* block_ids,
                                  const int64_t* token_ids, int64_t requests, int64_t tokens,
                                  int64_t table_width, int64_t block_size,
                                  int64_t* input_ids, int64_t* positions, int64_t* slot_mapping,
                                  int64_t* out_cu_seqlens_q, int64_t* out_query_starts,
                                  int64_t* context_lens, int64_t* block_tables, void* stream);

/* Fixed-shape decode metadata of a CUDA-graph bucket (the staging of
 * mini_engine/engine/cuda_graph.py:149-181 with the padding rows of :66-86):
 * rows r < *active take tokens[r], positions[r] and the block ids
 * block_ids[cu_blocks[r] : cu_blocks[r+1]]; the other rows get token 0,
 * position 0 and padding_pages[r] in column 0; all other columns are -1.
 * `active` is read on the device, so the launch can sit inside a graph. */
int minikv_build_decode_tables(const int64_t* active, const int64_t* tokens, const int64_t* positions,
                               const int64_t* cu_blocks, const int64_t* block_ids,
                               const int64_t* padding_pages, int64_t batch_size, int64_t max_blocks,
                               int64_t* input_ids, int64_t* out_positions, int64_t* block_tables,
                               void* stream);

/* ---------------------------------------------------------- decode step ---
 * Fused element-wise steps of the batch decode step around the paged-KV ops
 * (NativeQwen3.forward_decode_batch, mini_engine/model/native_qwen3.py:175-196
 * and :260-277).  FP16/BF16 only, like the reference's CUDA element-wise ops
 * (mini_engine/kernels/elementwise.py, bindings.cpp:209-214).  Every
 * intermediate is rounded to the 16-bit type where the eager torch path
 * rounds it (mini_engine/kernels/fallback.py:8-24).  Outputs must not overlap
 * inputs. */

/* out = RMSNorm(s) * weight over rows of `hidden` elements, where s = x, or
 * s = x + residual (rounded, and also written to sum_out) when residual is
 * given.  Replaces rms_norm / residual_rms_norm (elementwise.py:16-34) and,
 * fused into the next norm, residual_add (elementwise.py:37-44). */
int minikv_rms_norm(const void* x, const void* residual, const void* weight, void* out, void* sum_out,
                    int64_t rows, int64_t hidden, double eps, int dtype, void* stream);

/* out[r, j] = silu(gate_up[r, j]) * gate_up[r, inter + j]: silu_and_mul of a
 * fused gate|up projection (elementwise.py:47-54, native_qwen3.py:232-240). */
int minikv_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t inter, int dtype, void* stream);

/* Greedy next tokens: out[r] = index of the largest of x[r, 0 .. cols) (rows
 * row_stride elements apart; fp32, fp16 or bf16), where a NaN counts as the
 * largest and ties take the lowest index -- the semantics of the reference's
 * greedy sampler, logits.argmax(dim=-1) (mini_engine/sampling.py:14-22; its
 * CUDA variant sampling.cu:52-70).  Two chained launches: every warp of the
 * column slices of a row stores its best as a 64-bit key, then one warp per
 * row takes the largest key and turns it into the index.  `workspace` holds
 * minikv_argmax_workspace_bytes(rows, cols) bytes (16-byte aligned; scratch,
 * any contents); calls that may overlap on the GPU need separate workspaces.
 * No host synchronisation: capturable in a CUDA graph. */
int64_t minikv_argmax_workspace_bytes(int64_t rows, int64_t cols);
int minikv_argmax_rows(const void* x, int64_t rows, int64_t cols, int64_t row_stride, int dtype, void* workspace,
                       int64_t workspace_bytes, int64_t* out, void* stream);

/* Decode-step attention prologue in one launch over the fused q|k|v
 * projection rows (qkv[b, (q_heads + 2 kv_heads) * head_dim], row stride
 * qkv_stride elements): RMSNorm of every q and k head (q_weight, k_weight),
 * rotary embedding with cos/sin[b, head_dim/2], q written to q_out[b, q_heads,
 * head_dim], and the decode append of k (rotated) and v into the paged caches
 * at token_offsets[b] through block_tables (write_kv_cache_batch semantics,
 * data.cu:89-107: an out-of-range page skips the row).  Replaces q_norm,
 * k_norm, apply_rope and write_kv_cache_batch of native_qwen3.py:178-190.
 * head_dim 64, 128 or 256. */
int minikv_qk_rope_append(const void* qkv, int64_t qkv_stride, const void* q_weight, const void* k_weight,
                          const void* cos, const void* sin, void* q_out, void* key_cache, void* value_cache,
                          const int64_t* block_tables, const int64_t* token_offsets, int64_t batch,
                          int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                          int64_t block_size, int64_t table_width, double eps, int dtype, void* stream);

/* ---------------------------------------------------- fused projections ---
 * The dense projections of the batch decode step (FusedLinear, torch path
 * kernels/linear.py:116-130, i.e. y = x @ W^T with W [out, in] as in
 * nn.Linear) on the tcgen05 tensor cores, with the element-wise steps around
 * them fused in.  No counterpart in the reference's C++ API: these replace
 * the torch.mm + element-wise chains of native_qwen3.py:175-196 and
 * :232-277.  FP16/BF16; in_features a multiple of 64; x rows x_stride
 * elements apart (16-byte aligned).  The fp32 accumulation runs in the tensor
 * core's order and the split over in-features is summed in a fixed order, so
 * results are deterministic but not bit-equal to cuBLAS.
 *
 * Weights are passed packed (minikv_pack_linear, once at load time): the
 * [out, in] weight as [out / 128][in / 64] blocks of 128 rows x 64 elements,
 * each block contiguous and laid out as the tensor core reads it from shared
 * memory (16-byte chunk c of row r stored at chunk c ^ (r % 8)).
 *
 * RMSNorm prologue (ss_in != NULL): x is first normalised row by row,
 * T(T(x * rsqrt(ss / in_features + eps)) * norm_weight), where ss for token t
 * is the sum over j of ss_in[j * tokens + t], j < in_features / 128: the
 * partial sums of squares that minikv_linear_residual writes for its output.
 * in_features must then be a multiple of 128.  Outputs must not overlap
 * inputs. */

/* packed <- weight [out_features, in_features] (row-major, out_features a
 * multiple of 128) in the packed layout.  pair_offset > 0 packs a fused
 * gate|up weight (out_features = 2 pair_offset rows, pair_offset a multiple
 * of 64) for minikv_linear_silu_mul: block row-tile j then holds gate rows
 * [64 j, 64 j + 64) followed by up rows [pair_offset + 64 j, ...).  packed has
 * the size of weight and must not overlap it. */
int minikv_pack_linear(const void* weight, void* packed, int64_t out_features, int64_t in_features,
                       int64_t pair_offset, int dtype, void* stream);

/* out[t, n] = T(sum_k xn[t, k] weight[n, k]), out [tokens, out_features]
 * contiguous; out_features a multiple of 128. */
int minikv_linear(const void* x, int64_t x_stride, const float* ss_in, const void* norm_weight, double eps,
                  const void* packed_weight, void* out, int64_t tokens, int64_t in_features, int64_t out_features,
                  int dtype, void* stream);

/* out = T(T(x @ weight^T) + residual) (both [tokens, out_features]
 * contiguous) and, when ss_out != NULL, ss_out[j * tokens + t] = sum of
 * out[t, 128 j + i]^2 over i < 128 (fp32): the o projection or the down
 * projection with the residual add of native_qwen3.py:270-277, handing the
 * next RMSNorm its statistics. */
int minikv_linear_residual(const void* x, int64_t x_stride, const void* packed_weight, const void* residual,
                           void* out, float* ss_out, int64_t tokens, int64_t in_features, int64_t out_features,
                           int dtype, void* stream);

/* out[t, j] = T(T(silu(g)) * u) with g = T(xn @ gate^T)[t, j], u = T(xn @ up^T)[t, j],
 * where the fused weight cat(gate, up) [2 intermediate, in_features]
 * (enable_projection_fusion, native_qwen3.py:362-376) is packed with
 * pair_offset = intermediate; out [tokens, intermediate] contiguous,
 * intermediate a multiple of 64. */
int minikv_linear_silu_mul(const void* x, int64_t x_stride, const float* ss_in, const void* norm_weight, double eps,
                           const void* packed_gate_up, void* out, int64_t tokens, int64_t in_features,
                           int64_t intermediate, int dtype, void* stream);

/* The q|k|v projection (packed qkv weight [(q_heads + 2 kv_heads) * 128, in_features])
 * followed by what minikv_qk_rope_append does with its output: q/k RMSNorm,
 * rotary embedding (cos/sin [tokens, 64]), q to q_out [tokens, q_heads, 128],
 * K (rotated) and V appended at positions[t] through block_tables.  The
 * projection rows are never written to memory.  head_dim 128. */
int minikv_linear_qk_rope_append(const void* x, int64_t x_stride, const float* ss_in, const void* norm_weight,
                                 double eps, const void* packed_qkv, const void* q_weight, const void* k_weight,
                                 const void* cos, const void* sin, void* q_out, void* key_cache, void* value_cache,
                                 const int64_t* block_tables, const int64_t* positions, int64_t tokens,
                                 int64_t in_features, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                 int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MINIKV_H */
