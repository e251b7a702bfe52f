// Ragged causal paged prefill.
//
// Tensor-core route (prefill_tc.cu): bf16/fp16, head_dim 64 or 128, GQA group
// dividing 128, block_size a multiple of 8.  Over an FP8 pool it runs on a
// dense 16-bit copy of the pages the batch's tables reference (below).
//
// CUDA-core route (every other dtype / shape): each packed query token is turned
// into a one-token "decode request" -- its own query row, the page-table row
// of its request and the context length start + i + 1 it may attend
// (prefill.cu:112-123 of the reference computes the same per-token values) --
// and the balanced split-KV decode kernel runs over those tokens.  Tokens are
// processed in chunks of kPrefillChunk so the per-launch workspace stays
// bounded.
#include "common.cuh"
#include "prefill_tc.cu"

namespace minikv {

constexpr int64_t kPrefillChunk = 4096;

static int64_t prefill_core_workspace(int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                      int64_t block_size, int64_t table_width, int dtype, int sms,
                                      DecodePlan* plan_out) {
    const int64_t chunk = std::min(tokens, kPrefillChunk);
    DecodePlan plan;
    if (!make_decode_plan(chunk, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sms, &plan))
        return -1;
    if (plan_out) *plan_out = plan;
    return align256(chunk * 8) * 2 + plan.ws_bytes;
}

static int64_t prefill_workspace_bytes(int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                                       int64_t head_dim, int64_t block_size, int64_t table_width,
                                       int64_t max_query_len, int dtype, int sms) {
    (void)max_query_len;
    if (tokens <= 0) return 0;
    if (prefill_tc_supported(q_heads, kv_heads, head_dim, block_size, dtype, 1, tokens, requests)) return 0;
    return prefill_core_workspace(tokens, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sms,
                                  nullptr);
}

static int run_prefill(const void* q, const void* key_cache, const void* value_cache, const int64_t* cu_seqlens_q,
                       const int64_t* query_starts, const int64_t* block_tables, const int64_t* context_lens,
                       void* out, void* workspace, int64_t tokens, int64_t requests, int64_t q_heads,
                       int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                       int64_t table_width, int64_t max_query_len, int dtype, cudaStream_t stream) {
    (void)max_query_len;
    if (prefill_tc_supported(q_heads, kv_heads, head_dim, block_size, dtype, num_blocks, tokens, requests))
        return run_prefill_tc(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens, out,
                              tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                              dtype, stream);
    const int sms = sm_count();
    const int64_t chunk = std::min(tokens, kPrefillChunk);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int64_t* token_len = reinterpret_cast<int64_t*>(ws);
    int64_t* token_row = reinterpret_cast<int64_t*>(ws + align256(chunk * 8));
    void* decode_ws = ws + align256(chunk * 8) * 2;
    const int64_t es = dtype == 0 ? 4 : 2;
    const int64_t row_elems = q_heads * head_dim;
    for (int64_t t0 = 0; t0 < tokens; t0 += chunk) {
        const int64_t n = std::min(chunk, tokens - t0);
        DecodePlan plan;
        if (!make_decode_plan(n, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sms, &plan))
            return fail(MINIKV_EUNSUPPORTED, "paged prefill shape does not fit shared memory");
        const int64_t grid = std::min<int64_t>((n + 255) / 256, (int64_t)sms * 4);
        prefill_token_map_kernel<<<(unsigned)grid, 256, 0, stream>>>(cu_seqlens_q, query_starts, context_lens,
                                                                     requests, t0, n, table_width, block_size,
                                                                     token_len, token_row);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill token map");
        err = cudaMemsetAsync(decode_ws, 0, (size_t)decode_ticket_bytes(plan), stream);
        if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill ticket reset");
        const unsigned char* qn = static_cast<const unsigned char*>(q) + t0 * row_elems * es;
        unsigned char* on = static_cast<unsigned char*>(out) + t0 * row_elems * es;
        int rc = run_decode(qn, key_cache, value_cache, block_tables, token_len, token_row, on, decode_ws,
                            plan.ws_bytes, n, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                            dtype, stream);
        if (rc) return rc;
    }
    return MINIKV_OK;
}

// ------------------------------------------------------------- FP8 pools
// Three routes over an FP8 pool, the first that applies:
//  1. head_dim 128 and the tcgen05 kernel's shapes: the kernel stages the
//     pages' codes with TMA and converts them to fp16 in shared memory
//     (prefill_tc.cu, F8 != 0); no workspace.
//  2. the other tcgen05 shapes (head_dim 64): the dense copy below, then the
//     16-bit kernel;
//  3. the CUDA-core route (further below).
// Route 2: dequant_table_pages_kernel first writes a dense 16-bit copy of
// the pages the batch reads: table entry e = b * W + j becomes page e of the
// copy, with the codes converted exactly (every E4M3 and E5M2 value is an fp16
// and a bf16 value), and a remapped table holding e, or -1 where the entry is
// no page of the pool or lies past the request's context (those keys are
// masked either way).  The prefill then runs on the copy with the key scale
// folded into the softmax scale and the value scale into the output, the
// arithmetic of the FP8 decode.  Shared prefix pages are converted once per
// request that reads them.  Workspace: the two copies (W pages per request)
// and the remapped table; batches whose copies would pass
// kFp8PrefillCopyLimit take the CUDA-core route below instead.
constexpr int64_t kFp8PrefillCopyLimit = 8ll << 30;

template <typename T, bool E5M2>
__global__ void __launch_bounds__(256) dequant_table_pages_kernel(
    const unsigned char* __restrict__ kpool, const unsigned char* __restrict__ vpool,
    const int64_t* __restrict__ tables, const int64_t* __restrict__ context_lens, int64_t requests,
    int64_t width, int64_t num_blocks, int64_t block_size, int64_t page_bytes, T* __restrict__ kout,
    T* __restrict__ vout, int64_t* __restrict__ new_tables) {
    griddep_wait();
    griddep_launch_dependents();
    const int64_t chunks = page_bytes / 16;  // 16 codes per step
    const int64_t entries = requests * width;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < entries * chunks;
         q += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = q / chunks, ch = q - e * chunks;
        const int64_t b = e / width, j = e - b * width;
        const int64_t ctx = context_lens[b];
        const int64_t page = tables[e];
        const bool used = page >= 0 && page < num_blocks && ctx > 0 && j * block_size < ctx;
        if (ch == 0) new_tables[e] = used ? e : -1;
        if (!used) continue;
#pragma unroll
        for (int which = 0; which < 2; ++which) {
            const uint4 codes = ld_global_nc((which ? vpool : kpool) + page * page_bytes + ch * 16);
            const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
            uint32_t h[8];  // fp16 pairs of the 16 codes, in order
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                if (E5M2) {
                    h[2 * i] = byte_perm(w[i], 0u, 0x1404u);
                    h[2 * i + 1] = byte_perm(w[i], 0u, 0x3424u);
                } else {
                    h[2 * i] = e4m3x2_to_h2(w[i]);
                    h[2 * i + 1] = e4m3x2_to_h2(w[i] >> 16);
                }
            }
            uint4 o[2];
            uint32_t* ow = reinterpret_cast<uint32_t*>(o);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if constexpr (std::is_same<T, __half>::value) {
                    ow[i] = h[i];
                } else {  // exact: the fp16 value is a bf16 value
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
                    ow[i] = Elem<__nv_bfloat16>::pack(f.x, f.y);
                }
            }
            T* dst = (which ? vout : kout) + e * page_bytes + ch * 16;
            reinterpret_cast<uint4*>(dst)[0] = o[0];
            reinterpret_cast<uint4*>(dst)[1] = o[1];
        }
    }
}

// Bytes of the tensor-core route's copies for a batch, or -1 when it does not apply.
static int64_t prefill_fp8_copy_bytes(int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                                      int64_t head_dim, int64_t block_size, int64_t table_width, int dtype) {
    const int64_t entries = requests * table_width;
    if (entries <= 0 || !prefill_tc_supported(q_heads, kv_heads, head_dim, block_size, dtype, entries, tokens, requests))
        return -1;
    const int64_t copy = entries * block_size * kv_heads * head_dim * 2;  // one 16-bit pool
    const int64_t bytes = 2 * align256(copy) + align256(entries * 8);
    return bytes <= kFp8PrefillCopyLimit ? bytes : -1;
}

static int run_prefill_fp8_tc(const void* q, const void* key_cache, const void* value_cache,
                              const int64_t* cu_seqlens_q, const int64_t* query_starts, const int64_t* block_tables,
                              const int64_t* context_lens, void* out, void* workspace, int64_t tokens,
                              int64_t requests, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                              int64_t num_blocks, int64_t block_size, int64_t table_width, float k_scale,
                              float v_scale, bool e5m2, int dtype, cudaStream_t stream) {
    const int64_t entries = requests * table_width;
    const int64_t page_bytes = block_size * kv_heads * head_dim;  // fp8 bytes = 16-bit elements per page
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    unsigned char* kcopy = ws;
    unsigned char* vcopy = ws + align256(entries * page_bytes * 2);
    int64_t* tables = reinterpret_cast<int64_t*>(vcopy + align256(entries * page_bytes * 2));
    const int64_t work = entries * (page_bytes / 16);
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8));
    const unsigned char* kp = static_cast<const unsigned char*>(key_cache);
    const unsigned char* vp = static_cast<const unsigned char*>(value_cache);
    cudaError_t err;
    if (dtype == MINIKV_F16)
        err = e5m2 ? launch_chained(dequant_table_pages_kernel<__half, true>, dim3(grid), dim3(256), 0, stream, kp, vp,
                                    block_tables, context_lens, requests, table_width, num_blocks, block_size,
                                    page_bytes, reinterpret_cast<__half*>(kcopy), reinterpret_cast<__half*>(vcopy),
                                    tables)
                   : launch_chained(dequant_table_pages_kernel<__half, false>, dim3(grid), dim3(256), 0, stream, kp,
                                    vp, block_tables, context_lens, requests, table_width, num_blocks, block_size,
                                    page_bytes, reinterpret_cast<__half*>(kcopy), reinterpret_cast<__half*>(vcopy),
                                    tables);
    else
        err = e5m2 ? launch_chained(dequant_table_pages_kernel<__nv_bfloat16, true>, dim3(grid), dim3(256), 0, stream,
                                    kp, vp, block_tables, context_lens, requests, table_width, num_blocks, block_size,
                                    page_bytes, reinterpret_cast<__nv_bfloat16*>(kcopy),
                                    reinterpret_cast<__nv_bfloat16*>(vcopy), tables)
                   : launch_chained(dequant_table_pages_kernel<__nv_bfloat16, false>, dim3(grid), dim3(256), 0,
                                    stream, kp, vp, block_tables, context_lens, requests, table_width, num_blocks,
                                    block_size, page_bytes, reinterpret_cast<__nv_bfloat16*>(kcopy),
                                    reinterpret_cast<__nv_bfloat16*>(vcopy), tables);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill_fp8 page conversion");
    return run_prefill_tc(q, kcopy, vcopy, cu_seqlens_q, query_starts, tables, context_lens, out, tokens, requests,
                          q_heads, kv_heads, head_dim, entries, block_size, table_width, dtype, stream,
                          (double)k_scale, v_scale);
}

// Route 1 applies: head_dim 128 on the tcgen05 kernel's shapes.
static bool prefill_fp8_in_kernel(int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                                  int64_t head_dim, int64_t num_blocks, int64_t block_size, int dtype) {
    return head_dim == 128 &&
           prefill_tc_supported(q_heads, kv_heads, head_dim, block_size, dtype, num_blocks, tokens, requests);
}

// Workspace of the route a batch takes: none (route 1), the copies (route 2),
// or route 3's token map and decode workspace.  Route 3 runs the split-KV
// decode with the fp8 consumer, one row per query token, with the token map,
// chunking and workspace layout of the 16-bit CUDA-core route above; the
// decode plan is the fp8 pool's.
static int64_t prefill_fp8_workspace_bytes(int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                                           int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                           int64_t table_width, int dtype, int sms) {
    if (tokens <= 0) return 0;
    if (prefill_fp8_in_kernel(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, dtype)) return 0;
    const int64_t copy = prefill_fp8_copy_bytes(tokens, requests, q_heads, kv_heads, head_dim, block_size,
                                                table_width, dtype);
    if (copy >= 0) return copy;
    const int64_t chunk = std::min(tokens, kPrefillChunk);
    DecodePlan plan;
    if (!make_decode_plan(chunk, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sms, &plan, true))
        return -1;
    return align256(chunk * 8) * 2 + plan.ws_bytes;
}

static int run_prefill_fp8(const void* q, const void* key_cache, const void* value_cache,
                           const int64_t* cu_seqlens_q, const int64_t* query_starts, const int64_t* block_tables,
                           const int64_t* context_lens, void* out, void* workspace, int64_t tokens, int64_t requests,
                           int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                           int64_t block_size, int64_t table_width, float k_scale, float v_scale, bool e5m2,
                           int dtype, cudaStream_t stream) {
    if (prefill_fp8_in_kernel(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, dtype))
        return run_prefill_tc(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens, out,
                              tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                              dtype, stream, (double)k_scale, v_scale, e5m2 ? 2 : 1);
    if (prefill_fp8_copy_bytes(tokens, requests, q_heads, kv_heads, head_dim, block_size, table_width, dtype) >= 0)
        return run_prefill_fp8_tc(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens,
                                  out, workspace, tokens, requests, q_heads, kv_heads, head_dim, num_blocks,
                                  block_size, table_width, k_scale, v_scale, e5m2, dtype, stream);
    const int sms = sm_count();
    const int64_t chunk = std::min(tokens, kPrefillChunk);
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    int64_t* token_len = reinterpret_cast<int64_t*>(ws);
    int64_t* token_row = reinterpret_cast<int64_t*>(ws + align256(chunk * 8));
    unsigned char* decode_ws = ws + align256(chunk * 8) * 2;
    const int64_t row_bytes = q_heads * head_dim * 2;  // fp16/bf16 query and output
    for (int64_t t0 = 0; t0 < tokens; t0 += chunk) {
        const int64_t n = std::min(chunk, tokens - t0);
        DecodePlan plan;
        if (!make_decode_plan(n, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sms, &plan, true))
            return fail(MINIKV_EUNSUPPORTED, "paged prefill shape does not fit shared memory");
        const int64_t grid = std::min<int64_t>((n + 255) / 256, (int64_t)sms * 4);
        prefill_token_map_kernel<<<(unsigned)grid, 256, 0, stream>>>(cu_seqlens_q, query_starts, context_lens,
                                                                     requests, t0, n, table_width, block_size,
                                                                     token_len, token_row);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill_fp8 token map");
        err = cudaMemsetAsync(decode_ws, 0, (size_t)decode_ticket_bytes(plan), stream);
        if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill_fp8 ticket reset");
        const unsigned char* qn = static_cast<const unsigned char*>(q) + t0 * row_bytes;
        unsigned char* on = static_cast<unsigned char*>(out) + t0 * row_bytes;
        DecodeParams p = decode_params(qn, key_cache, value_cache, block_tables, token_len, token_row, on, decode_ws,
                                       n, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, plan);
        p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim) * (double)k_scale);
        p.out_scale = v_scale;
        err = dtype == MINIKV_F16 ? launch_decode_fp8<__half>(e5m2, (int)head_dim, p, plan, stream)
                                  : launch_decode_fp8<__nv_bfloat16>(e5m2, (int)head_dim, p, plan, stream);
        if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill_fp8 launch");
    }
    return MINIKV_OK;
}

}  // namespace minikv
