// Paged decode attention that allocates nothing: minikv_paged_decode_noalloc.
//
// Some callers cannot hand us scratch memory.  They cannot call cudaMalloc at
// the moment they need attention.  Examples: a host that is capturing a CUDA
// graph with a framework that owns every allocation; a serving loop that bans
// device allocation after start-up, because cudaMalloc can synchronise the
// device or fail under memory pressure in the middle of a request; a cgo / JNI
// host that has no device allocator of its own.  For them this entry point runs
// the same split-KV kernel as minikv_paged_decode, with its scratch (ticket
// counters, partial outputs, log-sum-exps) in the file-scope array below.
//
// Rules of use:
//  * the array holds kNoAllocScratchBytes (16 MiB) on every GPU that loads the
//    library, until the process exits; a call whose plan needs more scratch
//    fails with MINIKV_EINVAL before launching anything;
//  * all calls share the array and it keeps the previous call's contents: the
//    ticket counters, which must start at zero, are cleared on the call's
//    stream before every launch; two calls that overlap on the GPU (different
//    streams, or different host threads) race on the array and corrupt each
//    other's results, so callers must serialise them;
//  * the first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture on the device.  The cached address
//    belongs to the device's primary context: after cudaDeviceReset (or any
//    teardown of that context) it is stale, so a process that resets a device
//    must not call this entry point on it again.
#include <mutex>

#include "common.cuh"

namespace minikv {

constexpr int64_t kNoAllocScratchBytes = 16ll << 20;

// Device scratch of the no-allocation decode entry point.  In host code this
// name is only a stand-in for the symbol: its device address comes from
// cudaGetSymbolAddress (noalloc_scratch_ptr below).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  Returns nullptr (and sets the error message) on failure.
static void* noalloc_scratch_ptr() {
    constexpr int kMaxDevices = 64;
    static void* ptrs[kMaxDevices] = {nullptr};
    static std::mutex lock;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess || device < 0 || device >= kMaxDevices) {
        cuda_fail(err == cudaSuccess ? cudaErrorInvalidDevice : err, "minikv_paged_decode_noalloc device");
        return nullptr;
    }
    std::lock_guard<std::mutex> guard(lock);
    if (ptrs[device] == nullptr) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess || p == nullptr) {
            cuda_fail(err == cudaSuccess ? cudaErrorInvalidSymbol : err, "minikv_paged_decode_noalloc scratch lookup");
            return nullptr;
        }
        ptrs[device] = p;
    }
    return ptrs[device];
}

}  // namespace minikv

extern "C" int minikv_paged_decode_noalloc(const void* query, const void* key_cache, const void* value_cache,
                                           const int64_t* block_tables, const int64_t* context_lens, void* out,
                                           int64_t batch, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                           int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype,
                                           void* stream) {
    using namespace minikv;
    int rc = check_decode_shapes(batch, q_heads, kv_heads, head_dim, num_blocks, block_size, table_width, dtype);
    if (rc) return rc;
    MINIKV_REQUIRE(query && key_cache && value_cache && block_tables && context_lens && out, MINIKV_EINVAL,
                   "null pointer argument");
    MINIKV_REQUIRE(aligned16(query) && aligned16(key_cache) && aligned16(value_cache) && aligned16(out),
                   MINIKV_EINVAL, "query, caches and output must be 16-byte aligned");
    DecodePlan plan;
    if (!make_decode_plan(batch, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sm_count(), &plan))
        return fail(MINIKV_EUNSUPPORTED, "decode shape does not fit shared memory (batch too large?)");
    if (plan.ws_bytes > kNoAllocScratchBytes)
        return fail(MINIKV_EINVAL, "minikv_paged_decode_noalloc needs " + std::to_string(plan.ws_bytes) +
                                       " bytes of scratch; its built-in buffer holds " +
                                       std::to_string(kNoAllocScratchBytes) +
                                       " (use minikv_paged_decode with a caller workspace)");
    void* scratch = noalloc_scratch_ptr();
    if (scratch == nullptr) return MINIKV_ECUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The ticket counters must be zero at launch (the buffer is shared by all calls).
    cudaError_t err = cudaMemsetAsync(static_cast<unsigned char*>(scratch) + plan.ws_tickets, 0,
                                      (size_t)decode_ticket_bytes(plan), s);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_decode_noalloc ticket reset");
    const DecodeParams p = decode_params(query, key_cache, value_cache, block_tables, context_lens, nullptr, out,
                                         static_cast<unsigned char*>(scratch), batch, q_heads, kv_heads, head_dim,
                                         num_blocks, block_size, table_width, plan);
    err = launch_decode(dtype, (int)head_dim, p, plan, s);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_decode_noalloc launch");
    return MINIKV_OK;
}
