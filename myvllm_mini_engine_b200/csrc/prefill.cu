// Ragged causal paged prefill.
//
// Tensor-core route (prefill_tc.cu): bf16/fp16, head_dim 64 or 128, GQA group
// dividing 128, block_size a multiple of 8.
//
// CUDA-core route (every other dtype / shape, and every FP8 pool): each packed query token is turned
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

// FP8 pool: the CUDA-core route with the fp8 decode consumer (the tensor-core
// route stages 16-bit pages only).  Same token map, chunking and workspace
// layout as above; the decode plan is the fp8 pool's.
static int64_t prefill_fp8_workspace_bytes(int64_t tokens, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                           int64_t block_size, int64_t table_width, int dtype, int sms) {
    if (tokens <= 0) return 0;
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
