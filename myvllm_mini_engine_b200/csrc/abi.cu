// extern "C" entry points of libminikv (declared in include/minikv.h).
//
// Each entry point checks its arguments (returning MINIKV_EINVAL with a
// message, never throwing across the ABI), picks the kernel instantiation and
// launches on the caller's stream.  Messages reuse the wording of the
// reference's TORCH_CHECKs (mini_engine/kernels/csrc/bindings.cpp:152-184,
// data.cu:209-237, prefill.cu:200-233) where a check has a counterpart there.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/minikv.h"
#include "common.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& message) {
    g_last_error = message;
    return code;
}

int cuda_fail(cudaError_t err, const char* where) {
    return fail(MINIKV_ECUDA, std::string(where) + ": " + cudaGetErrorString(err));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_dtype(int dtype) { return dtype == MINIKV_F32 || dtype == MINIKV_F16 || dtype == MINIKV_BF16; }

bool valid_head_dim(int64_t d) {
    return d == 16 || d == 32 || d == 64 || d == 80 || d == 96 || d == 128 || d == 192 || d == 256;
}

int elem_bytes(int dtype) { return dtype == MINIKV_F32 ? 4 : 2; }

int sm_count() {
    static int cached[64] = {0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
    if (cached[device] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        cached[device] = n > 0 ? n : 148;
    }
    return cached[device];
}

// Raise a kernel's opt-in dynamic shared-memory limit on the current device to at
// least `bytes`.  `configured` is the kernel's per-device record of the limit
// already set (64 entries).  The check and the set happen under one lock and the
// limit only ever grows, so host threads launching the same kernel with
// different plans never leave it below a plan that passed the check.
std::mutex g_smem_attribute_lock;

template <typename Kernel>
cudaError_t ensure_smem_limit(Kernel kernel, int bytes, int* configured) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return err;
    const bool tracked = device >= 0 && device < 64;
    std::lock_guard<std::mutex> guard(g_smem_attribute_lock);
    if (tracked && configured[device] >= bytes) return cudaSuccess;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess && tracked) configured[device] = bytes;
    return err;
}

#define MINIKV_REQUIRE(cond, code, msg) \
    do {                                \
        if (!(cond)) return fail(code, msg); \
    } while (0)

}  // namespace

#include "kv_write.cu"
#include "decode.cu"
#include "decode_fp8.cu"
#include "metadata.cu"
#include "prefill.cu"
#include "decode_step.cu"
#include "proj.cu"

using namespace minikv;

extern "C" {

int minikv_abi_version(void) { return MINIKV_ABI_VERSION; }

#ifndef MINIKV_SOURCE_HASH
#define MINIKV_SOURCE_HASH "unknown"
#endif
// The marker prefix lets the build recipe read the hash from the file without loading it.
static const char kSourceHash[] = "minikv-source-hash:" MINIKV_SOURCE_HASH;

const char* minikv_source_hash(void) { return kSourceHash + sizeof("minikv-source-hash:") - 1; }

const char* minikv_last_error(void) { return g_last_error.c_str(); }

int minikv_device_status(unsigned int* status, int clear, void* stream) {
    MINIKV_REQUIRE(status != nullptr, MINIKV_EINVAL, "status pointer is null");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaStreamSynchronize(s);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_device_status");
    err = cudaMemcpyFromSymbol(status, g_status, sizeof(unsigned int));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_device_status");
    if (clear) {
        const unsigned int zero = 0;
        err = cudaMemcpyToSymbol(g_status, &zero, sizeof(unsigned int));
        if (err != cudaSuccess) return cuda_fail(err, "minikv_device_status");
    }
    return MINIKV_OK;
}

int minikv_set_wait_limit(uint64_t limit_ns, void* stream) {
    MINIKV_REQUIRE(limit_ns > 0, MINIKV_EINVAL, "the wait limit must be positive");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned long long value = limit_ns;
    cudaError_t err = cudaStreamSynchronize(s);  // no kernel of the stream runs while the limit changes
    if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_space_wait_limit_ns, &value, sizeof(value));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_set_wait_limit");
    return MINIKV_OK;
}

// ------------------------------------------------------------------- decode
static int check_decode_shapes(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                               int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype) {
    MINIKV_REQUIRE(valid_dtype(dtype), MINIKV_EINVAL, "FP32/FP16/BF16 required");
    MINIKV_REQUIRE(batch > 0 && q_heads > 0 && num_blocks > 0 && kv_heads > 0, MINIKV_EINVAL,
                   "empty batch/heads/cache");
    MINIKV_REQUIRE(block_size > 0, MINIKV_EINVAL, "block size mismatch");
    MINIKV_REQUIRE(q_heads % kv_heads == 0, MINIKV_EINVAL, "head dimension or GQA mismatch");
    MINIKV_REQUIRE(valid_head_dim(head_dim), MINIKV_EINVAL, "supported head_dim: 16,32,64,80,96,128,192,256");
    MINIKV_REQUIRE(table_width > 0, MINIKV_EINVAL, "invalid block table");
    MINIKV_REQUIRE(table_width * block_size <= 1048576, MINIKV_EINVAL, "maximum table capacity is 1M tokens");
    MINIKV_REQUIRE(batch * q_heads <= 2147483647, MINIKV_EINVAL, "batch/head product too large");
    MINIKV_REQUIRE(num_blocks * block_size <= 2147483647, MINIKV_EINVAL, "KV pool exceeds 2^31 token rows");
    return MINIKV_OK;
}

int64_t minikv_paged_decode_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                            int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                            int64_t table_width, int dtype) {
    if (check_decode_shapes(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype))
        return -1;
    DecodePlan plan;
    if (!make_decode_plan(batch, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sm_count(), &plan))
        return -1;
    return plan.ws_bytes;
}

int minikv_paged_decode(const void* query, const void* key_cache, const void* value_cache,
                        const int64_t* block_tables, const int64_t* context_lens, void* out,
                        void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                        int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                        int64_t table_width, int dtype, void* stream) {
    int rc = check_decode_shapes(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(query && key_cache && value_cache && block_tables && context_lens && out, MINIKV_EINVAL,
                   "null pointer argument");
    MINIKV_REQUIRE(aligned16(query) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out),
                   MINIKV_EINVAL, "query, caches and output must be 16-byte aligned");
    return run_decode(query, key_cache, value_cache, block_tables, context_lens, nullptr, out, workspace,
                      workspace_bytes, batch, q_heads, kv_heads, head_dim, num_blocks, block_size,
                      table_width, dtype, static_cast<cudaStream_t>(stream));
}

int minikv_paged_decode_chained(const void* query, const void* key_cache, const void* value_cache,
                                const int64_t* block_tables, const int64_t* context_lens, void* out,
                                void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                                int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                int64_t table_width, int dtype, void* stream) {
    int rc = check_decode_shapes(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(query && key_cache && value_cache && block_tables && context_lens && out, MINIKV_EINVAL,
                   "null pointer argument");
    MINIKV_REQUIRE(aligned16(query) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out),
                   MINIKV_EINVAL, "query, caches and output must be 16-byte aligned");
    return run_decode(query, key_cache, value_cache, block_tables, context_lens, nullptr, out, workspace,
                      workspace_bytes, batch, q_heads, kv_heads, head_dim, num_blocks, block_size,
                      table_width, dtype, static_cast<cudaStream_t>(stream), true);
}

int minikv_paged_decode_append(const void* query, const void* key_cache, const void* value_cache,
                               const int64_t* block_tables, const int64_t* token_offsets, const void* key,
                               const void* value, void* out, void* workspace, int64_t workspace_bytes,
                               int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                               int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype, int chained,
                               void* stream) {
    int rc = check_decode_shapes(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(query && key_cache && value_cache && block_tables && token_offsets && key && value && out,
                   MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(query) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out) &&
                       aligned16(key) && aligned16(value),
                   MINIKV_EINVAL, "query, caches, new K/V rows and output must be 16-byte aligned");
    return run_decode(query, key_cache, value_cache, block_tables, token_offsets, nullptr, out, workspace,
                      workspace_bytes, batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                      dtype, static_cast<cudaStream_t>(stream), chained != 0, key, value);
}

// ---------------------------------------------------------------- KV writes
static int check_rows(const void* kc, const void* vc, const void* k, const void* v, int64_t kv_heads,
                      int64_t head_dim, int64_t k_stride, int64_t v_stride, int dtype) {
    MINIKV_REQUIRE(valid_dtype(dtype), MINIKV_EINVAL, "KV cache requires FP32/FP16/BF16");
    MINIKV_REQUIRE(kv_heads > 0 && head_dim > 0, MINIKV_EINVAL, "K/V head shape mismatch");
    const int64_t row_bytes = kv_heads * head_dim * elem_bytes(dtype);
    MINIKV_REQUIRE(row_bytes % 16 == 0, MINIKV_EINVAL, "KV row (kv_heads*head_dim) must be a multiple of 16 bytes");
    MINIKV_REQUIRE(k_stride >= kv_heads * head_dim && v_stride >= kv_heads * head_dim, MINIKV_EINVAL,
                   "K/V token stride smaller than a row");
    MINIKV_REQUIRE((k_stride * elem_bytes(dtype)) % 16 == 0 && (v_stride * elem_bytes(dtype)) % 16 == 0,
                   MINIKV_EINVAL, "K/V token stride must be a multiple of 16 bytes");
    MINIKV_REQUIRE(kc && vc && k && v, MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(kc) && aligned16(vc) && aligned16(k) && aligned16(v), MINIKV_EINVAL,
                   "KV tensors must be 16-byte aligned");
    return MINIKV_OK;
}

int minikv_kv_scatter_slots(void* key_cache, void* value_cache, const int64_t* slot_mapping, const void* key,
                            const void* value, int64_t tokens, int64_t num_blocks, int64_t block_size,
                            int64_t kv_heads, int64_t head_dim, int64_t key_token_stride,
                            int64_t value_token_stride, int dtype, void* stream) {
    MINIKV_REQUIRE(tokens >= 0, MINIKV_EINVAL, "packed KV slots must be int64 [tokens]");
    MINIKV_REQUIRE(num_blocks > 0 && block_size > 0, MINIKV_EINVAL, "packed KV cache must be nonempty");
    if (tokens == 0) return MINIKV_OK;
    int rc = check_rows(key_cache, value_cache, key, value, kv_heads, head_dim, key_token_stride,
                        value_token_stride, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(slot_mapping != nullptr, MINIKV_EINVAL, "null slot_mapping");
    const int64_t es = elem_bytes(dtype);
    cudaError_t err = launch_write_rows(key_cache, value_cache, key, value, tokens, kv_heads * head_dim * es,
                                        key_token_stride * es, value_token_stride * es,
                                        SlotRows{slot_mapping, num_blocks * block_size},
                                        static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_kv_scatter_slots launch");
    return MINIKV_OK;
}

// ----------------------------------------------------------- FP8 KV pool
static bool valid_scale(float s) { return std::isfinite(s) && s > 0.f; }

static int check_fp8_decode(int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                            int64_t block_size, int64_t table_width, int dtype) {
    MINIKV_REQUIRE(dtype == MINIKV_F16 || dtype == MINIKV_BF16, MINIKV_EINVAL,
                   "an fp8 KV pool needs an FP16/BF16 query");
    MINIKV_REQUIRE(fp8_head_dim(head_dim), MINIKV_EINVAL, "fp8 KV pool: supported head_dim: 32,64,96,128,192,256");
    return check_decode_shapes(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype);
}

int64_t minikv_paged_decode_fp8_workspace_bytes(int64_t batch, int64_t q_heads, int64_t kv_heads,
                                                int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                                int64_t table_width, int dtype) {
    if (check_fp8_decode(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype)) return -1;
    DecodePlan plan;
    if (!make_decode_plan(batch, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sm_count(), &plan, true))
        return -1;
    return plan.ws_bytes;
}

static int run_decode_fp8(const void* query, const void* key_cache, const void* value_cache,
                          const int64_t* block_tables, const int64_t* lens, const void* key, const void* value,
                          void* out, void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                          int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                          int64_t table_width, float k_scale, float v_scale, int fp8_format, int dtype, bool chained,
                          void* stream) {
    MINIKV_REQUIRE(fp8_format == MINIKV_FP8_E4M3 || fp8_format == MINIKV_FP8_E5M2, MINIKV_EINVAL,
                   "fp8 format must be E4M3 or E5M2");
    int rc = check_fp8_decode(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(valid_scale(k_scale) && valid_scale(v_scale), MINIKV_EINVAL,
                   "fp8 KV scales must be finite and positive");
    MINIKV_REQUIRE(query && key_cache && value_cache && block_tables && lens && out, MINIKV_EINVAL,
                   "null pointer argument");
    MINIKV_REQUIRE(aligned16(query) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out),
                   MINIKV_EINVAL, "query, caches and output must be 16-byte aligned");
    DecodePlan plan;
    if (!make_decode_plan(batch, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sm_count(), &plan, true))
        return fail(MINIKV_EUNSUPPORTED, "decode shape does not fit shared memory (batch too large?)");
    MINIKV_REQUIRE(workspace != nullptr && workspace_bytes >= plan.ws_bytes && aligned16(workspace),
                   MINIKV_EINVAL, "decode workspace too small or misaligned");
    DecodeParams p = decode_params(query, key_cache, value_cache, block_tables, lens, nullptr, out,
                                   static_cast<unsigned char*>(workspace), batch, q_heads, kv_heads, head_dim,
                                   num_blocks, block_size, table_width, plan);
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim) * (double)k_scale);
    p.out_scale = v_scale;
    p.early_prologue = chained ? 1 : 0;
    if (key != nullptr) {  // fused append: lens holds the token offsets
        p.append = 1;
        p.new_k = key;
        p.new_v = value;
        p.k_inv = 1.0f / k_scale;  // the factors of the quantising slot scatter
        p.v_inv = 1.0f / v_scale;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool e5m2 = fp8_format == MINIKV_FP8_E5M2;
    const cudaError_t err = dtype == MINIKV_F16 ? launch_decode_fp8<__half>(e5m2, (int)head_dim, p, plan, s)
                                                : launch_decode_fp8<__nv_bfloat16>(e5m2, (int)head_dim, p, plan, s);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_decode_fp8 launch");
    return MINIKV_OK;
}

int minikv_paged_decode_fp8(const void* query, const void* key_cache, const void* value_cache,
                            const int64_t* block_tables, const int64_t* context_lens, void* out,
                            void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                            int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                            int64_t table_width, float k_scale, float v_scale, int fp8_format, int dtype,
                            void* stream) {
    return run_decode_fp8(query, key_cache, value_cache, block_tables, context_lens, nullptr, nullptr, out,
                          workspace, workspace_bytes, batch, q_heads, kv_heads, head_dim, num_blocks, block_size,
                          table_width, k_scale, v_scale, fp8_format, dtype, false, stream);
}

int minikv_paged_decode_fp8_append(const void* query, const void* key_cache, const void* value_cache,
                                   const int64_t* block_tables, const int64_t* token_offsets, const void* key,
                                   const void* value, void* out, void* workspace, int64_t workspace_bytes,
                                   int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                   int64_t num_blocks, int64_t block_size, int64_t table_width, float k_scale,
                                   float v_scale, int fp8_format, int dtype, int chained, void* stream) {
    MINIKV_REQUIRE(key && value && token_offsets, MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(key) && aligned16(value), MINIKV_EINVAL, "new K/V rows must be 16-byte aligned");
    return run_decode_fp8(query, key_cache, value_cache, block_tables, token_offsets, key, value, out, workspace,
                          workspace_bytes, batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                          k_scale, v_scale, fp8_format, dtype, chained != 0, stream);
}

int minikv_kv_scatter_slots_fp8(void* key_cache, void* value_cache, const int64_t* slot_mapping, const void* key,
                                const void* value, int64_t tokens, int64_t num_blocks, int64_t block_size,
                                int64_t kv_heads, int64_t head_dim, int64_t key_token_stride,
                                int64_t value_token_stride, float k_scale, float v_scale, int fp8_format, int dtype,
                                void* stream) {
    MINIKV_REQUIRE(fp8_format == MINIKV_FP8_E4M3 || fp8_format == MINIKV_FP8_E5M2, MINIKV_EINVAL,
                   "fp8 format must be E4M3 or E5M2");
    MINIKV_REQUIRE(tokens >= 0, MINIKV_EINVAL, "packed KV slots must be int64 [tokens]");
    MINIKV_REQUIRE(num_blocks > 0 && block_size > 0, MINIKV_EINVAL, "packed KV cache must be nonempty");
    MINIKV_REQUIRE(valid_dtype(dtype), MINIKV_EINVAL, "packed KV requires FP32/FP16/BF16");
    MINIKV_REQUIRE(valid_scale(k_scale) && valid_scale(v_scale), MINIKV_EINVAL,
                   "fp8 KV scales must be finite and positive");
    MINIKV_REQUIRE(kv_heads > 0 && head_dim > 0, MINIKV_EINVAL, "K/V head shape mismatch");
    const int64_t row_elems = kv_heads * head_dim;
    MINIKV_REQUIRE(row_elems % 16 == 0, MINIKV_EINVAL, "fp8 KV row (kv_heads*head_dim) must be a multiple of 16");
    MINIKV_REQUIRE(key_token_stride >= row_elems && value_token_stride >= row_elems, MINIKV_EINVAL,
                   "K/V token stride smaller than a row");
    if (tokens == 0) return MINIKV_OK;
    MINIKV_REQUIRE(key_cache && value_cache && key && value && slot_mapping, MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(key_cache) && aligned16(value_cache), MINIKV_EINVAL, "KV caches must be 16-byte aligned");
    const float k_inv = 1.0f / k_scale, v_inv = 1.0f / v_scale;
    const bool e5m2 = fp8_format == MINIKV_FP8_E5M2;
    const int64_t capacity = num_blocks * block_size;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err;
    if (dtype == MINIKV_F32)
        err = launch_quantize_slots<float>(key_cache, value_cache, key, value, slot_mapping, tokens, capacity,
                                           row_elems, key_token_stride, value_token_stride, k_inv, v_inv, e5m2, s);
    else if (dtype == MINIKV_F16)
        err = launch_quantize_slots<__half>(key_cache, value_cache, key, value, slot_mapping, tokens, capacity,
                                            row_elems, key_token_stride, value_token_stride, k_inv, v_inv, e5m2, s);
    else
        err = launch_quantize_slots<__nv_bfloat16>(key_cache, value_cache, key, value, slot_mapping, tokens,
                                                   capacity, row_elems, key_token_stride, value_token_stride, k_inv,
                                                   v_inv, e5m2, s);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_kv_scatter_slots_fp8 launch");
    return MINIKV_OK;
}

int minikv_kv_append_batch(void* key_cache, void* value_cache, const int64_t* block_tables,
                           const int64_t* token_offsets, const void* key, const void* value, int64_t batch,
                           int64_t table_width, int64_t num_blocks, int64_t block_size, int64_t kv_heads,
                           int64_t head_dim, int64_t key_token_stride, int64_t value_token_stride, int dtype,
                           void* stream) {
    MINIKV_REQUIRE(batch >= 0 && table_width >= 0, MINIKV_EINVAL, "batch table shape mismatch");
    MINIKV_REQUIRE(num_blocks > 0 && block_size > 0, MINIKV_EINVAL, "batch block size mismatch");
    if (batch == 0) return MINIKV_OK;
    MINIKV_REQUIRE(table_width > 0, MINIKV_EINVAL, "batch table shape mismatch");
    int rc = check_rows(key_cache, value_cache, key, value, kv_heads, head_dim, key_token_stride,
                        value_token_stride, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(block_tables && token_offsets, MINIKV_EINVAL, "null metadata pointer");
    const int64_t es = elem_bytes(dtype);
    cudaError_t err = launch_write_rows(key_cache, value_cache, key, value, batch, kv_heads * head_dim * es,
                                        key_token_stride * es, value_token_stride * es,
                                        AppendRows{block_tables, token_offsets, table_width, num_blocks, block_size},
                                        static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_kv_append_batch launch");
    return MINIKV_OK;
}

int minikv_kv_write_range(void* key_cache, void* value_cache, const int64_t* block_ids, int64_t num_ids,
                          int64_t token_offset, const void* key, const void* value, int64_t tokens,
                          int64_t num_blocks, int64_t block_size, int64_t kv_heads, int64_t head_dim,
                          int64_t key_token_stride, int64_t value_token_stride, int dtype, void* stream) {
    MINIKV_REQUIRE(num_blocks > 0 && block_size > 0, MINIKV_EINVAL, "block size mismatch");
    MINIKV_REQUIRE(token_offset >= 0 && tokens >= 0 && token_offset + tokens <= num_ids * block_size,
                   MINIKV_EINVAL, "KV write exceeds block table");
    if (tokens == 0) return MINIKV_OK;
    int rc = check_rows(key_cache, value_cache, key, value, kv_heads, head_dim, key_token_stride,
                        value_token_stride, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(block_ids != nullptr, MINIKV_EINVAL, "null block ids");
    const int64_t es = elem_bytes(dtype);
    cudaError_t err = launch_write_rows(key_cache, value_cache, key, value, tokens, kv_heads * head_dim * es,
                                        key_token_stride * es, value_token_stride * es,
                                        RangeRows{block_ids, num_ids, token_offset, num_blocks, block_size},
                                        static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_kv_write_range launch");
    return MINIKV_OK;
}

int minikv_copy_blocks(void* key_pool, void* value_pool, const int64_t* pairs, int64_t num_pairs,
                       int64_t num_layers, int64_t num_blocks, int64_t block_elems, int dtype, void* stream) {
    MINIKV_REQUIRE(valid_dtype(dtype), MINIKV_EINVAL, "KV pool requires FP32/FP16/BF16");
    MINIKV_REQUIRE(num_pairs >= 0 && num_layers > 0 && num_blocks > 0 && block_elems > 0, MINIKV_EINVAL,
                   "copy_blocks shape mismatch");
    if (num_pairs == 0) return MINIKV_OK;
    const int64_t page_bytes = block_elems * elem_bytes(dtype);
    MINIKV_REQUIRE(page_bytes % 16 == 0, MINIKV_EINVAL, "page must be a multiple of 16 bytes");
    MINIKV_REQUIRE(key_pool && value_pool && pairs, MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(key_pool) && aligned16(value_pool), MINIKV_EINVAL, "pools must be 16-byte aligned");
    cudaError_t err = launch_copy_blocks(key_pool, value_pool, pairs, num_pairs, num_layers, num_blocks, page_bytes,
                                         static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_copy_blocks launch");
    return MINIKV_OK;
}

// ------------------------------------------------------------------ prefill
static int check_prefill(int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                         int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype) {
    MINIKV_REQUIRE(valid_dtype(dtype), MINIKV_EINVAL, "paged prefill requires FP32/FP16/BF16");
    MINIKV_REQUIRE(block_size > 0 && num_blocks > 0 && kv_heads > 0 && head_dim > 0, MINIKV_EINVAL,
                   "paged prefill cache/block size mismatch");
    MINIKV_REQUIRE(q_heads > 0 && q_heads % kv_heads == 0 && valid_head_dim(head_dim), MINIKV_EINVAL,
                   "paged prefill GQA/head_dim mismatch");
    MINIKV_REQUIRE(tokens >= 0 && requests >= 0 && table_width >= 0, MINIKV_EINVAL,
                   "paged prefill metadata shape mismatch");
    MINIKV_REQUIRE(tokens * q_heads <= 2147483647, MINIKV_EINVAL, "too many paged prefill rows");
    MINIKV_REQUIRE(num_blocks * block_size <= 2147483647, MINIKV_EINVAL, "KV pool exceeds 2^31 token rows");
    return MINIKV_OK;
}

int64_t minikv_paged_prefill_workspace_bytes(int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                                             int64_t head_dim, int64_t num_blocks, int64_t block_size,
                                             int64_t table_width, int64_t max_query_len, int dtype) {
    if (check_prefill(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype))
        return -1;
    return prefill_workspace_bytes(tokens, requests, q_heads, kv_heads, head_dim, block_size, table_width,
                                   max_query_len, dtype, sm_count());
}

int minikv_paged_prefill(const void* q, const void* key_cache, const void* value_cache,
                         const int64_t* cu_seqlens_q, const int64_t* query_starts, const int64_t* block_tables,
                         const int64_t* context_lens, void* out, void* workspace, int64_t workspace_bytes,
                         int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                         int64_t num_blocks, int64_t block_size, int64_t table_width, int64_t max_query_len,
                         int dtype, void* stream) {
    int rc = check_prefill(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                           dtype);
    if (rc) return rc;
    if (tokens == 0) return MINIKV_OK;
    MINIKV_REQUIRE(requests > 0 && table_width > 0, MINIKV_EINVAL, "paged prefill metadata shape mismatch");
    MINIKV_REQUIRE(q && key_cache && value_cache && cu_seqlens_q && query_starts && block_tables && context_lens &&
                       out,
                   MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(q) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out), MINIKV_EINVAL,
                   "paged prefill tensors must be 16-byte aligned");
    const int64_t need = prefill_workspace_bytes(tokens, requests, q_heads, kv_heads, head_dim, block_size,
                                                 table_width, max_query_len, dtype, sm_count());
    MINIKV_REQUIRE(need >= 0, MINIKV_EUNSUPPORTED, "paged prefill shape does not fit shared memory");
    MINIKV_REQUIRE(workspace_bytes >= need && (need == 0 || (workspace && aligned16(workspace))), MINIKV_EINVAL,
                   "paged prefill workspace too small or misaligned");
    return run_prefill(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens, out,
                       workspace, tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                       max_query_len, dtype, static_cast<cudaStream_t>(stream));
}

int64_t minikv_paged_prefill_fp8_workspace_bytes(int64_t tokens, int64_t requests, int64_t q_heads,
                                                 int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                                                 int64_t block_size, int64_t table_width, int64_t max_query_len,
                                                 int dtype) {
    (void)max_query_len;
    if (check_prefill(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype))
        return -1;
    if ((dtype != MINIKV_F16 && dtype != MINIKV_BF16) || !fp8_head_dim(head_dim)) return -1;
    return prefill_fp8_workspace_bytes(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size,
                                       table_width, dtype, sm_count());
}

int minikv_paged_prefill_fp8(const void* q, const void* key_cache, const void* value_cache,
                             const int64_t* cu_seqlens_q, const int64_t* query_starts, const int64_t* block_tables,
                             const int64_t* context_lens, void* out, void* workspace, int64_t workspace_bytes,
                             int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                             int64_t num_blocks, int64_t block_size, int64_t table_width, int64_t max_query_len,
                             float k_scale, float v_scale, int fp8_format, int dtype, void* stream) {
    (void)max_query_len;
    MINIKV_REQUIRE(fp8_format == MINIKV_FP8_E4M3 || fp8_format == MINIKV_FP8_E5M2, MINIKV_EINVAL,
                   "fp8 format must be E4M3 or E5M2");
    int rc = check_prefill(tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width,
                           dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(dtype == MINIKV_F16 || dtype == MINIKV_BF16, MINIKV_EINVAL,
                   "an fp8 KV pool needs an FP16/BF16 query");
    MINIKV_REQUIRE(fp8_head_dim(head_dim), MINIKV_EINVAL, "fp8 KV pool: supported head_dim: 32,64,96,128,192,256");
    MINIKV_REQUIRE(valid_scale(k_scale) && valid_scale(v_scale), MINIKV_EINVAL,
                   "fp8 KV scales must be finite and positive");
    if (tokens == 0) return MINIKV_OK;
    MINIKV_REQUIRE(requests > 0 && table_width > 0, MINIKV_EINVAL, "paged prefill metadata shape mismatch");
    MINIKV_REQUIRE(q && key_cache && value_cache && cu_seqlens_q && query_starts && block_tables && context_lens &&
                       out,
                   MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(q) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out), MINIKV_EINVAL,
                   "paged prefill tensors must be 16-byte aligned");
    const int64_t need = prefill_fp8_workspace_bytes(tokens, requests, q_heads, kv_heads, head_dim, num_blocks,
                                                     block_size, table_width, dtype, sm_count());
    MINIKV_REQUIRE(need >= 0, MINIKV_EUNSUPPORTED, "paged prefill shape does not fit shared memory");
    MINIKV_REQUIRE(workspace_bytes >= need && (need == 0 || (workspace && aligned16(workspace))), MINIKV_EINVAL,
                   "paged prefill workspace too small or misaligned");
    return run_prefill_fp8(q, key_cache, value_cache, cu_seqlens_q, query_starts, block_tables, context_lens, out,
                           workspace, tokens, requests, q_heads, kv_heads, head_dim, num_blocks, block_size,
                           table_width, k_scale, v_scale, fp8_format == MINIKV_FP8_E5M2, dtype,
                           static_cast<cudaStream_t>(stream));
}

// ----------------------------------------------------------------- metadata
int minikv_build_prefill_metadata(const int64_t* query_starts, const int64_t* cu_seqlens_q, const int64_t* cu_blocks,
                                  const int64_t* block_ids, const int64_t* token_ids, int64_t requests,
                                  int64_t tokens, int64_t table_width, int64_t block_size, int64_t* input_ids,
                                  int64_t* positions, int64_t* slot_mapping, int64_t* out_cu_seqlens_q,
                                  int64_t* out_query_starts, int64_t* context_lens, int64_t* block_tables,
                                  void* stream) {
    MINIKV_REQUIRE(requests > 0 && tokens >= 0 && table_width > 0 && block_size > 0, MINIKV_EINVAL,
                   "prefill metadata shape mismatch");
    MINIKV_REQUIRE(query_starts && cu_seqlens_q && cu_blocks && block_ids && (token_ids || tokens == 0) &&
                       (input_ids || tokens == 0) && (positions || tokens == 0) && (slot_mapping || tokens == 0) &&
                       out_cu_seqlens_q && out_query_starts && context_lens && block_tables,
                   MINIKV_EINVAL, "null pointer argument");
    const int64_t grid = std::min<int64_t>(requests, (int64_t)sm_count() * 4);
    prefill_metadata_kernel<<<(unsigned)grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        query_starts, cu_seqlens_q, cu_blocks, block_ids, token_ids, requests, table_width, block_size, input_ids,
        positions, slot_mapping, out_cu_seqlens_q, out_query_starts, context_lens, block_tables);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, "minikv_build_prefill_metadata launch");
    return MINIKV_OK;
}

int minikv_build_decode_tables(const int64_t* active, const int64_t* tokens, const int64_t* positions,
                               const int64_t* cu_blocks, const int64_t* block_ids, const int64_t* padding_pages,
                               int64_t batch_size, int64_t max_blocks, int64_t* input_ids, int64_t* out_positions,
                               int64_t* block_tables, void* stream) {
    MINIKV_REQUIRE(batch_size > 0 && max_blocks > 0, MINIKV_EINVAL, "decode bucket shape must be positive");
    MINIKV_REQUIRE(active && tokens && positions && cu_blocks && block_ids && padding_pages && input_ids &&
                       out_positions && block_tables,
                   MINIKV_EINVAL, "null pointer argument");
    const int64_t grid = std::min<int64_t>(batch_size, (int64_t)sm_count() * 4);
    decode_tables_kernel<<<(unsigned)grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        active, tokens, positions, cu_blocks, block_ids, padding_pages, batch_size, max_blocks, input_ids,
        out_positions, block_tables);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, "minikv_build_decode_tables launch");
    return MINIKV_OK;
}

// ---------------------------------------------------------------- decode step
int minikv_rms_norm(const void* x, const void* residual, const void* weight, void* out, void* sum_out,
                    int64_t rows, int64_t hidden, double eps, int dtype, void* stream) {
    MINIKV_REQUIRE(dtype == MINIKV_F16 || dtype == MINIKV_BF16, MINIKV_EUNSUPPORTED, "FP16/BF16 required");
    MINIKV_REQUIRE(rows >= 0 && hidden > 0 && hidden % 8 == 0 && hidden <= 8192, MINIKV_EINVAL,
                   "hidden size must be a positive multiple of 8 and at most 8192");
    MINIKV_REQUIRE(x && weight && out && (residual == nullptr) == (sum_out == nullptr), MINIKV_EINVAL,
                   "null pointer argument (residual and sum_out go together)");
    MINIKV_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(out) && (!residual || aligned16(residual)) &&
                       (!sum_out || aligned16(sum_out)),
                   MINIKV_EINVAL, "tensors must be 16-byte aligned");
    cudaError_t err = launch_rms_norm(dtype, x, residual, weight, out, sum_out, rows, (int)hidden, (float)eps,
                                      static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_rms_norm launch");
    return MINIKV_OK;
}

int minikv_silu_mul(const void* gate_up, void* out, int64_t rows, int64_t inter, int dtype, void* stream) {
    MINIKV_REQUIRE(dtype == MINIKV_F16 || dtype == MINIKV_BF16, MINIKV_EUNSUPPORTED, "FP16/BF16 required");
    MINIKV_REQUIRE(rows >= 0 && inter > 0 && inter % 8 == 0, MINIKV_EINVAL,
                   "intermediate size must be a positive multiple of 8");
    MINIKV_REQUIRE(gate_up && out, MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(gate_up) && aligned16(out), MINIKV_EINVAL, "tensors must be 16-byte aligned");
    cudaError_t err = launch_silu_mul(dtype, gate_up, out, rows, inter, sm_count(), static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_silu_mul launch");
    return MINIKV_OK;
}

int64_t minikv_argmax_workspace_bytes(int64_t rows, int64_t cols) {
    if (rows <= 0 || cols <= 0 || rows > 65535) return -1;
    return argmax_workspace_bytes(rows, cols, sm_count());
}

int minikv_argmax_rows(const void* x, int64_t rows, int64_t cols, int64_t row_stride, int dtype, void* workspace,
                       int64_t workspace_bytes, int64_t* out, void* stream) {
    MINIKV_REQUIRE(valid_dtype(dtype), MINIKV_EINVAL, "FP32/FP16/BF16 required");
    MINIKV_REQUIRE(rows > 0 && rows <= 65535 && cols > 0 && cols < (1ll << 31) && row_stride >= cols, MINIKV_EINVAL,
                   "argmax needs 1..65535 rows of 1..2^31-1 columns within the row stride");
    MINIKV_REQUIRE(x && out && workspace, MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(workspace_bytes >= argmax_workspace_bytes(rows, cols, sm_count()) && aligned16(workspace),
                   MINIKV_EINVAL, "argmax workspace too small or misaligned");
    cudaError_t err = launch_argmax(dtype, x, rows, cols, row_stride, workspace, out, sm_count(),
                                    static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_argmax_rows launch");
    return MINIKV_OK;
}

int minikv_qk_rope_append(const void* qkv, int64_t qkv_stride, const void* q_weight, const void* k_weight,
                          const void* cos, const void* sin, void* q_out, void* key_cache, void* value_cache,
                          const int64_t* block_tables, const int64_t* token_offsets, int64_t batch, int64_t q_heads,
                          int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                          int64_t table_width, double eps, int dtype, void* stream) {
    MINIKV_REQUIRE(dtype == MINIKV_F16 || dtype == MINIKV_BF16, MINIKV_EUNSUPPORTED, "FP16/BF16 required");
    MINIKV_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, MINIKV_EUNSUPPORTED,
                   "head_dim must be 64, 128 or 256");
    MINIKV_REQUIRE(batch >= 0 && q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0 && num_blocks > 0 &&
                       block_size > 0 && table_width > 0,
                   MINIKV_EINVAL, "query heads must be divisible by KV heads");
    MINIKV_REQUIRE(qkv_stride >= (q_heads + 2 * kv_heads) * head_dim && qkv_stride % 8 == 0, MINIKV_EINVAL,
                   "qkv rows must hold q, k and v heads and start on 16 bytes");
    MINIKV_REQUIRE(qkv && q_weight && k_weight && cos && sin && q_out && key_cache && value_cache && block_tables &&
                       token_offsets,
                   MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(qkv) && aligned16(q_weight) && aligned16(k_weight) && aligned16(cos) &&
                       aligned16(sin) && aligned16(q_out) && aligned16(key_cache) && aligned16(value_cache),
                   MINIKV_EINVAL, "tensors must be 16-byte aligned");
    QkRopeParams p;
    p.qkv = qkv; p.q_weight = q_weight; p.k_weight = k_weight; p.cos = cos; p.sin = sin; p.q_out = q_out;
    p.key_cache = key_cache; p.value_cache = value_cache; p.tables = block_tables; p.offsets = token_offsets;
    p.batch = batch; p.qkv_stride = qkv_stride; p.width = table_width; p.num_blocks = num_blocks;
    p.block_size = block_size; p.q_heads = (int)q_heads; p.kv_heads = (int)kv_heads; p.eps = (float)eps;
    cudaError_t err = launch_qk_rope_append(dtype, p, (int)head_dim, sm_count(), static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_qk_rope_append launch");
    return MINIKV_OK;
}

// ------------------------------------------------------ fused projections
int minikv_pack_linear(const void* weight, void* packed, int64_t out_features, int64_t in_features,
                       int64_t pair_offset, int dtype, void* stream) {
    MINIKV_REQUIRE(dtype == MINIKV_F16 || dtype == MINIKV_BF16, MINIKV_EUNSUPPORTED, "FP16/BF16 required");
    MINIKV_REQUIRE(in_features > 0 && in_features % 64 == 0 && out_features > 0 && out_features % 128 == 0 &&
                       out_features * in_features < (1ll << 40),
                   MINIKV_EINVAL, "packing needs out_features % 128 == 0 and in_features % 64 == 0");
    MINIKV_REQUIRE(pair_offset == 0 || (pair_offset % 64 == 0 && 2 * pair_offset == out_features), MINIKV_EINVAL,
                   "a paired (gate|up) weight has 2 * pair_offset rows, pair_offset a multiple of 64");
    MINIKV_REQUIRE(weight && packed && aligned16(weight) && aligned16(packed), MINIKV_EINVAL,
                   "weights must be 16-byte aligned");
    cudaError_t err = launch_pack_linear(dtype, weight, packed, out_features, in_features, pair_offset, sm_count(),
                                         static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_pack_linear launch");
    return MINIKV_OK;
}

int minikv_linear(const void* x, int64_t x_stride, const float* ss_in, const void* norm_weight, double eps,
                  const void* packed_weight, void* out, int64_t tokens, int64_t in_features, int64_t out_features,
                  int dtype, void* stream) {
    ProjParams p;
    int rc = proj_setup(x, x_stride, packed_weight, tokens, in_features, out_features, ss_in, norm_weight, dtype, &p);
    if (rc != MINIKV_OK) return rc;
    MINIKV_REQUIRE(out_features % 128 == 0, MINIKV_EINVAL, "out_features must be a multiple of 128");
    MINIKV_REQUIRE(out && aligned16(out), MINIKV_EINVAL, "out must be 16-byte aligned");
    if (tokens == 0) return MINIKV_OK;
    p.out_features = (int)out_features;
    p.eps = (float)eps;
    p.out = out;
    p.out_stride = out_features;
    cudaError_t err = launch_proj<kEpiStore>(dtype, ss_in != nullptr, p, out_features / 128,
                                             static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_linear launch");
    return MINIKV_OK;
}

int minikv_linear_residual(const void* x, int64_t x_stride, const void* packed_weight, const void* residual,
                           void* out, float* ss_out, int64_t tokens, int64_t in_features, int64_t out_features, int dtype,
                           void* stream) {
    ProjParams p;
    int rc = proj_setup(x, x_stride, packed_weight, tokens, in_features, out_features, nullptr, nullptr, dtype, &p);
    if (rc != MINIKV_OK) return rc;
    MINIKV_REQUIRE(out_features % 128 == 0, MINIKV_EINVAL, "out_features must be a multiple of 128");
    MINIKV_REQUIRE(residual && out && aligned16(residual) && aligned16(out), MINIKV_EINVAL,
                   "residual and out must be 16-byte aligned");
    if (tokens == 0) return MINIKV_OK;
    p.out_features = (int)out_features;
    p.out = out;
    p.out_stride = out_features;
    p.residual = residual;
    p.residual_stride = out_features;
    p.ss_out = ss_out;
    cudaError_t err = launch_proj<kEpiResidual>(dtype, false, p, out_features / 128,
                                                static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_linear_residual launch");
    return MINIKV_OK;
}

int minikv_linear_silu_mul(const void* x, int64_t x_stride, const float* ss_in, const void* norm_weight, double eps,
                           const void* packed_gate_up, void* out, int64_t tokens, int64_t in_features,
                           int64_t intermediate, int dtype, void* stream) {
    ProjParams p;
    MINIKV_REQUIRE(intermediate > 0 && intermediate % 64 == 0 && intermediate < (1ll << 30), MINIKV_EINVAL,
                   "intermediate size must be a positive multiple of 64");
    int rc = proj_setup(x, x_stride, packed_gate_up, tokens, in_features, 2 * intermediate, ss_in, norm_weight,
                        dtype, &p);
    if (rc != MINIKV_OK) return rc;
    MINIKV_REQUIRE(out && aligned16(out), MINIKV_EINVAL, "out must be 16-byte aligned");
    if (tokens == 0) return MINIKV_OK;
    p.out_features = (int)intermediate;
    p.gate_offset = (int)intermediate;
    p.eps = (float)eps;
    p.out = out;
    p.out_stride = intermediate;
    cudaError_t err = launch_proj<kEpiSiluMul>(dtype, ss_in != nullptr, p, intermediate / 64,
                                               static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_linear_silu_mul launch");
    return MINIKV_OK;
}

int minikv_linear_qk_rope_append(const void* x, int64_t x_stride, const float* ss_in, const void* norm_weight,
                                 double eps, const void* packed_qkv, const void* q_weight, const void* k_weight,
                                 const void* cos, const void* sin, void* q_out, void* key_cache, void* value_cache,
                                 const int64_t* block_tables, const int64_t* positions, int64_t tokens,
                                 int64_t in_features, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                 int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype,
                                 void* stream) {
    MINIKV_REQUIRE(head_dim == 128, MINIKV_EUNSUPPORTED, "the fused q|k|v projection needs head_dim 128");
    MINIKV_REQUIRE(q_heads > 0 && kv_heads > 0 && q_heads % kv_heads == 0 && q_heads + 2 * kv_heads < 65536 &&
                       num_blocks > 0 && block_size > 0 && table_width > 0,
                   MINIKV_EINVAL, "query heads must be divisible by KV heads");
    const int64_t rows = (q_heads + 2 * kv_heads) * head_dim;
    ProjParams p;
    int rc = proj_setup(x, x_stride, packed_qkv, tokens, in_features, rows, ss_in, norm_weight, dtype, &p);
    if (rc != MINIKV_OK) return rc;
    MINIKV_REQUIRE(q_weight && k_weight && cos && sin && q_out && key_cache && value_cache && block_tables &&
                       positions,
                   MINIKV_EINVAL, "null pointer argument");
    MINIKV_REQUIRE(aligned16(q_weight) && aligned16(k_weight) && aligned16(cos) && aligned16(sin) &&
                       aligned16(q_out) && aligned16(key_cache) && aligned16(value_cache),
                   MINIKV_EINVAL, "tensors must be 16-byte aligned");
    if (tokens == 0) return MINIKV_OK;
    p.out_features = (int)rows;
    p.eps = (float)eps;
    p.out = q_out;
    p.q_weight = q_weight;
    p.k_weight = k_weight;
    p.cos = cos;
    p.sin = sin;
    p.key_cache = key_cache;
    p.value_cache = value_cache;
    p.tables = block_tables;
    p.positions = positions;
    p.width = table_width;
    p.num_blocks = num_blocks;
    p.block_size = block_size;
    p.q_heads = (int)q_heads;
    p.kv_heads = (int)kv_heads;
    cudaError_t err = launch_proj<kEpiQkRope>(dtype, ss_in != nullptr, p, q_heads + 2 * kv_heads,
                                              static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return cuda_fail(err, "minikv_linear_qk_rope_append launch");
    return MINIKV_OK;
}

}  // extern "C"

// The no-allocation decode entry point (its scratch array and its set-up live in
// that file; it uses check_decode_shapes above).
#include "decode_noalloc.cu"
