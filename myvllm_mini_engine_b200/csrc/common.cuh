// Shared device helpers for the paged-KV kernels (sm_100a).
//
// * element traits: 16-byte vectors of fp32 / fp16 / bf16 <-> fp32 registers;
// * mbarrier + 1-D bulk-copy (TMA engine) wrappers in inline PTX;
// * bounded waits: every spin on an mbarrier polls with try_wait and gives up
//   after a limit of %globaltimer time (2 s), records an error bit in the device
//   status word and lets the kernel run to its end.  Three kinds:
//     mbar_wait        data waits (copies or MMAs landing);
//     mbar_wait_space  a producer waiting for consumers to free a ring slot;
//                      its limit is g_space_wait_limit_ns, which the host can
//                      shorten (minikv_set_wait_limit) to exercise this path;
//     mbar_drain       a thread waiting for the copies or MMAs it issued itself
//                      before its CTA exits (no early give-up).
//   After a failed space wait a producer issues nothing more and drains what
//   it has issued; after a failed data wait a consumer skips that stage's
//   data (it may still be landing) but keeps its arrivals, so the CTA always
//   exits with no copy or MMA in flight.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace minikv {

// Device status word, read and cleared by minikv_device_status().
// Bit values are listed in include/minikv.h (MINIKV_STATUS_*).  The library
// is one translation unit (abi.cu includes the kernel files), so the word is
// defined here once.
__device__ unsigned int g_status = 0;

__device__ __forceinline__ void raise_status(unsigned int bit) { atomicOr(&g_status, bit); }

constexpr unsigned int kStatusWaitTimeout = 1u;

// ----------------------------------------------------------------- element traits
template <typename T> struct Elem;
template <> struct Elem<float> {
    static constexpr int kPerVec = 4;  // elements per 16-byte vector
    __device__ static __forceinline__ void load(const uint4& v, float* f) {
        f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
    }
    __device__ static __forceinline__ uint4 store(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                          __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
    __device__ static __forceinline__ float to_float(float x) { return x; }
    __device__ static __forceinline__ float from_float(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
    static constexpr int kPerVec = 8;
    __device__ static __forceinline__ void unpack(uint32_t w, float* f) {
        // bf16 is the high half of an fp32: widening is a shift / mask.
        f[0] = __uint_as_float(w << 16);
        f[1] = __uint_as_float(w & 0xffff0000u);
    }
    __device__ static __forceinline__ void load(const uint4& v, float* f) {
        unpack(v.x, f); unpack(v.y, f + 2); unpack(v.z, f + 4); unpack(v.w, f + 6);
    }
    __device__ static __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ static __forceinline__ uint4 store(const float* f) {
        return make_uint4(pack(f[0], f[1]), pack(f[2], f[3]), pack(f[4], f[5]), pack(f[6], f[7]));
    }
    __device__ static __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
    __device__ static __forceinline__ __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
    static constexpr int kPerVec = 8;
    __device__ static __forceinline__ void unpack(uint32_t w, float* f) {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        float2 x = __half22float2(h);
        f[0] = x.x; f[1] = x.y;
    }
    __device__ static __forceinline__ void load(const uint4& v, float* f) {
        unpack(v.x, f); unpack(v.y, f + 2); unpack(v.z, f + 4); unpack(v.w, f + 6);
    }
    __device__ static __forceinline__ uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ static __forceinline__ uint4 store(const float* f) {
        return make_uint4(pack(f[0], f[1]), pack(f[2], f[3]), pack(f[4], f[5]), pack(f[6], f[7]));
    }
    __device__ static __forceinline__ float to_float(__half x) { return __half2float(x); }
    __device__ static __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};

// ----------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy before first use.
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}

// One polling probe of the phase with the given parity (no suspend-time hint:
// the call returns after a short, hardware-defined interval at the latest).
// Non-blocking probe of a phase (returns at once).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return done != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done) : "r"(smem_addr(bar)), "r"(parity) : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint64_t kWaitCheckNs = 200000ull;       // 200 us: from here on, check for another timeout

// Limit of the space waits (mbar_wait_space); minikv_set_wait_limit changes it.
__device__ unsigned long long g_space_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ bool status_timed_out() {
    return (*reinterpret_cast<volatile unsigned int*>(&g_status) & kStatusWaitTimeout) != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and sets
// the status bit) if the phase did not complete within `limit`; with
// `early_out`, a wait that has lasted kWaitCheckNs also gives up when another
// wait already timed out, so a broken pipeline costs one limit, not one per
// wait.  Callers then carry on so that the kernel reaches its end.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint64_t limit, bool early_out) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    for (;;) {
        // one probe between clock reads: a probe can suspend the thread for a
        // hardware-defined interval, so limits below a microsecond stay meaningful
        if (mbar_try_wait(bar, parity)) return true;
        const uint64_t waited = global_ns() - start;
        if (waited > limit) break;
        if (early_out && waited > kWaitCheckNs && status_timed_out()) return false;
    }
    raise_status(kStatusWaitTimeout);
    return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, kWaitLimitNs, true);
}

// The space-wait limit, read once per kernel by the producers.
__device__ __forceinline__ uint64_t space_wait_limit() {
    return *reinterpret_cast<volatile unsigned long long*>(&g_space_wait_limit_ns);
}

__device__ __forceinline__ bool mbar_wait_space(uint64_t* bar, uint32_t parity, uint64_t limit) {
    if (limit >= kWaitCheckNs) return mbar_wait_for(bar, parity, limit, true);
    // a short limit (a test of the timeout path): non-blocking probes between clock reads, so the
    // limit is not hidden by the suspend interval of a blocking probe
    if (mbar_test_wait(bar, parity)) return true;
    const uint64_t start = global_ns();
    while (!mbar_test_wait(bar, parity)) {
        if (global_ns() - start > limit) {
            raise_status(kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
    return mbar_wait_for(bar, parity, kWaitLimitNs, false);
}

// 1-D bulk copy global -> shared through the TMA engine; completion is
// counted in bytes on `bar`.  dst, src and bytes must be 16-byte multiples.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy) : "memory");
}

// L2 eviction-priority policies for bulk loads.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// --------------------------------------------- programmatic dependent launch
// Kernels of a launch chain are launched with programmatic stream
// serialization (launch_chained): such a kernel may start while the previous
// kernel on the stream is still running, so it must execute griddep_wait()
// before it touches anything that kernel (or an earlier one) writes.  A kernel
// that calls griddep_launch_dependents() lets the next chained kernel start
// early.  Launched without the attribute, both instructions are no-ops.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                  Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

__device__ __forceinline__ uint4 ld_global_nc(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

template <int N> struct Log2 { static constexpr int value = 1 + Log2<N / 2>::value; };
template <> struct Log2<1> { static constexpr int value = 0; };

}  // namespace minikv
