// Element-wise steps of the Qwen3 batch decode step that surround the paged-KV
// ops (mini_engine/model/native_qwen3.py:175-196 attention, :260-277 layer),
// fused so that a 28-layer step is a few launches per layer:
//
//   * rms_norm_kernel        RMSNorm of rows, optionally after a residual add
//                            (fallback.py:8-10; elementwise.py:24-31, 37-42);
//   * silu_mul_kernel        SiLU(gate) * up over a fused gate|up row
//                            (fallback.py:23-24; native_qwen3.py:232-240);
//   * qk_rope_append_kernel  per-head q/k RMSNorm, rotary embedding and the
//                            decode KV append in one pass over the fused
//                            q|k|v projection (native_qwen3.py:178-190;
//                            fallback.py:13-20; data.py:67-81).
//
// All three are chained launches (programmatic dependent launch): each waits
// for the previous kernel at entry, so only its launch latency overlaps.
//
// Rounding follows the eager reference: every torch op there returns the
// 16-bit input type, so each intermediate (the sum, the normalised row, the
// product with the weight, each rotary product and their sum) is rounded to
// T here at the same point; reductions and transcendental functions run in
// fp32, as torch's opmath does.
#include <climits>

#include "common.cuh"

namespace minikv {

template <typename T> struct Narrow;
template <> struct Narrow<__nv_bfloat16> {
    __device__ static __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <> struct Narrow<__half> {
    __device__ static __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};

// Sum over the CTA (blockDim.x a multiple of 32, at most 1024).
__device__ __forceinline__ float block_sum(float v, float* scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    if ((threadIdx.x & 31) == 0) scratch[warp] = v;
    __syncthreads();
    float total = 0.f;
    for (int w = 0; w < warps; ++w) total += scratch[w];
    return total;
}

// One CTA per row of `hidden` elements (hidden % 8 == 0, hidden <= 8 * blockDim.x * kVecs).
//   s   = T(x + residual)           (when residual != nullptr; written to sum_out)
//   out = T(T(s * rsqrt(mean(s^2) + eps)) * weight)
template <typename T, int kVecs>
__global__ void __launch_bounds__(256) rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ residual,
                                                       const T* __restrict__ weight, T* __restrict__ out,
                                                       T* __restrict__ sum_out, int hidden, float eps) {
    __shared__ float scratch[32];
    griddep_wait();
    griddep_launch_dependents();
    const int64_t row = blockIdx.x;
    const int vecs = hidden / 8;
    const uint4* xs = reinterpret_cast<const uint4*>(x + row * hidden);
    const uint4* rs = residual ? reinterpret_cast<const uint4*>(residual + row * hidden) : nullptr;
    float v[kVecs][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kVecs; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < vecs) {
            Elem<T>::load(ld_global_nc(xs + c), v[i]);
            if (rs) {
                float r[8];
                Elem<T>::load(ld_global_nc(rs + c), r);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[i][j] = Narrow<T>::round(v[i][j] + r[j]);
                reinterpret_cast<uint4*>(sum_out + row * hidden)[c] = Elem<T>::store(v[i]);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
        }
    }
    const float inv = rsqrtf(block_sum(ss, scratch) / (float)hidden + eps);
    const uint4* ws = reinterpret_cast<const uint4*>(weight);
    uint4* os = reinterpret_cast<uint4*>(out + row * hidden);
#pragma unroll
    for (int i = 0; i < kVecs; ++i) {
        const int c = threadIdx.x + i * blockDim.x;
        if (c < vecs) {
            float w[8];
            Elem<T>::load(ld_global_nc(ws + c), w);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[i][j] = Narrow<T>::round(v[i][j] * inv) * w[j];
            os[c] = Elem<T>::store(v[i]);
        }
    }
}

// out[r, j] = T(T(silu(g)) * u) with g = gate_up[r, j], u = gate_up[r, inter + j]
// (inter % 8 == 0).  silu(g) = g / (1 + exp(-g)) in fp32.
template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T* __restrict__ gate_up, T* __restrict__ out,
                                                       int64_t rows, int64_t inter) {
    griddep_wait();
    griddep_launch_dependents();
    const int64_t vecs_per_row = inter / 8;
    const int64_t total = rows * vecs_per_row;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / vecs_per_row, c = i % vecs_per_row;
        const uint4* row = reinterpret_cast<const uint4*>(gate_up + r * 2 * inter);
        float g[8], u[8];
        Elem<T>::load(ld_global_nc(row + c), g);
        Elem<T>::load(ld_global_nc(row + vecs_per_row + c), u);
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = Narrow<T>::round(g[j] / (1.0f + expf(-g[j]))) * u[j];
        reinterpret_cast<uint4*>(out + r * inter)[c] = Elem<T>::store(g);
    }
}

// Load / store kE consecutive 16-bit elements (kE = 2, 4 or 8).
template <typename T, int kE> struct Lane;
template <typename T> struct Lane<T, 2> {
    __device__ static void load(const T* p, float* f) { Elem<T>::unpack(*reinterpret_cast<const uint32_t*>(p), f); }
    __device__ static void store(T* p, const float* f) { *reinterpret_cast<uint32_t*>(p) = Elem<T>::pack(f[0], f[1]); }
};
template <typename T> struct Lane<T, 4> {
    __device__ static void load(const T* p, float* f) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        Elem<T>::unpack(v.x, f); Elem<T>::unpack(v.y, f + 2);
    }
    __device__ static void store(T* p, const float* f) {
        *reinterpret_cast<uint2*>(p) = make_uint2(Elem<T>::pack(f[0], f[1]), Elem<T>::pack(f[2], f[3]));
    }
};
template <typename T> struct Lane<T, 8> {
    __device__ static void load(const T* p, float* f) { Elem<T>::load(*reinterpret_cast<const uint4*>(p), f); }
    __device__ static void store(T* p, const float* f) { *reinterpret_cast<uint4*>(p) = Elem<T>::store(f); }
};

struct QkRopeParams {
    const void* qkv;          // [batch, (q_heads + 2 kv_heads) * D] row stride qkv_stride elements
    const void* q_weight;     // [D] q_norm weight
    const void* k_weight;     // [D] k_norm weight
    const void* cos;          // [batch, D/2]
    const void* sin;          // [batch, D/2]
    void* q_out;              // [batch, q_heads, D]
    void* key_cache;          // [num_blocks, block_size, kv_heads, D]
    void* value_cache;
    const int64_t* tables;    // [batch, width]
    const int64_t* offsets;   // [batch] position of the appended token
    int64_t batch, qkv_stride, width, num_blocks, block_size;
    int q_heads, kv_heads;
    float eps;
};

// One warp per (request, head) for the q heads and the kv heads.  Lane l holds
// elements [l*kE, (l+1)*kE); the rotary partner of element i < D/2 is i + D/2,
// held by lane l ^ 16.
template <typename T, int D>
__global__ void __launch_bounds__(256) qk_rope_append_kernel(const QkRopeParams p) {
    constexpr int kE = D / 32;
    constexpr int kHalf = D / 2;
    griddep_wait();
    griddep_launch_dependents();  // the decode of the same layer may start its prologue
    const int lane = threadIdx.x & 31;
    const int64_t heads = p.q_heads + p.kv_heads;
    const int64_t jobs = p.batch * heads;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t job = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); job < jobs; job += warps) {
        const int64_t b = job / heads;
        const int h = (int)(job % heads);
        const bool is_q = h < p.q_heads;
        const T* row = static_cast<const T*>(p.qkv) + b * p.qkv_stride;
        const T* src = row + (int64_t)h * D + lane * kE;  // k heads follow the q heads
        float x[kE], w[kE];
        Lane<T, kE>::load(src, x);
        Lane<T, kE>::load(static_cast<const T*>(is_q ? p.q_weight : p.k_weight) + lane * kE, w);
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < kE; ++j) ss += x[j] * x[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss / (float)D + p.eps);
#pragma unroll
        for (int j = 0; j < kE; ++j) x[j] = Narrow<T>::round(Narrow<T>::round(x[j] * inv) * w[j]);
        // rotary: first half  y1 = T(T(x1 c) - T(x2 s)); second half y2 = T(T(x1 s) + T(x2 c))
        float c[kE], s[kE], y[kE];
        const int64_t angle = b * kHalf + (int64_t)(lane & 15) * kE;
        Lane<T, kE>::load(static_cast<const T*>(p.cos) + angle, c);
        Lane<T, kE>::load(static_cast<const T*>(p.sin) + angle, s);
        const bool first = lane < 16;
#pragma unroll
        for (int j = 0; j < kE; ++j) {
            const float other = __shfl_xor_sync(0xffffffffu, x[j], 16);
            if (first) {
                y[j] = Narrow<T>::round(Narrow<T>::round(x[j] * c[j]) - Narrow<T>::round(other * s[j]));
            } else {
                y[j] = Narrow<T>::round(Narrow<T>::round(other * s[j]) + Narrow<T>::round(x[j] * c[j]));
            }
        }
        if (is_q) {
            Lane<T, kE>::store(static_cast<T*>(p.q_out) + (b * p.q_heads + h) * D + lane * kE, y);
            continue;
        }
        // decode append of this kv head's K (rotated) and V (as projected): data.cu:89-107 guards
        const int kvh = h - p.q_heads;
        const int64_t logical = p.offsets[b];
        if (logical < 0) continue;
        const int64_t index = logical / p.block_size;
        if (index >= p.width) continue;
        const int64_t page = p.tables[b * p.width + index];
        if (page < 0 || page >= p.num_blocks) continue;
        const int64_t dst = ((page * p.block_size + logical % p.block_size) * p.kv_heads + kvh) * D + lane * kE;
        Lane<T, kE>::store(static_cast<T*>(p.key_cache) + dst, y);
        float v[kE];
        Lane<T, kE>::load(row + (int64_t)(p.q_heads + p.kv_heads + kvh) * D + lane * kE, v);
        Lane<T, kE>::store(static_cast<T*>(p.value_cache) + dst, v);
    }
}

// ------------------------------------------------------------ greedy argmax
// out[r] = index of the largest value of row r: a NaN counts as the largest
// and ties take the lowest index, the semantics of torch.argmax (the
// reference's greedy sampler, mini_engine/sampling.py:14-22).  Two chained
// launches.  argmax_rows_kernel: CTA (s, r) scans columns [s * per, (s + 1) *
// per) of row r with 16-byte loads (four in flight per thread); each warp
// stores its best as a 64-bit key that orders (value, then lower index): the
// high word is the value's bits made monotonic (every NaN the largest), the
// low word the complemented column.  argmax_keys_kernel (one warp per row,
// after the first launch has ended) takes the largest key of the row's slots
// and turns it into the index.
__device__ __forceinline__ bool argmax_before(float a, int ai, float b, int bi) {
    // does (a, ai) win over (b, bi)?
    const bool an = a != a, bn = b != b;
    if (an || bn) return an && (!bn || ai < bi);
    return a > b || (a == b && ai < bi);
}

struct ArgmaxBest {
    float v;
    int i;  // column (columns < 2^31); INT_MAX: none yet
    __device__ __forceinline__ void take(float x, int j) {
        if (argmax_before(x, j, v, i)) {
            v = x;
            i = j;
        }
    }
};

// max with NaN propagation (a NaN operand gives NaN)
__device__ __forceinline__ float max_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t hi = (v != v) ? 0xffffffffu : ((u & 0x80000000u) ? ~u : (u | 0x80000000u));
    return ((unsigned long long)hi << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}

template <typename T, bool kVec>
__global__ void __launch_bounds__(256) argmax_rows_kernel(const T* __restrict__ x, int64_t cols, int64_t stride,
                                                          int64_t per, unsigned long long* __restrict__ slots) {
    griddep_wait();
    griddep_launch_dependents();
    const int s = blockIdx.x;
    const int64_t r = blockIdx.y;
    const T* row = x + r * stride;
    const int64_t lo = (int64_t)s * per, hi = min(cols, lo + per);
    ArgmaxBest best{-INFINITY, INT_MAX};
    if (kVec) {  // the row start and `per` are 16-byte multiples: [lo, hiv) in 16-byte vectors of kV elements
        constexpr int kV = Elem<T>::kPerVec, kInFlight = 4;  // loads issued before any is consumed
        const int64_t hiv = lo + ((hi - lo) / kV) * kV;
        const int64_t step = kV * (int64_t)blockDim.x;
        for (int64_t c0 = lo + kV * (int64_t)threadIdx.x; c0 < hiv; c0 += kInFlight * step) {
            uint4 v[kInFlight];
#pragma unroll
            for (int u = 0; u < kInFlight; ++u)
                if (c0 + u * step < hiv) v[u] = *reinterpret_cast<const uint4*>(row + c0 + u * step);
#pragma unroll
            for (int u = 0; u < kInFlight; ++u) {
                if (c0 + u * step >= hiv) break;
                float f[kV];
                Elem<T>::load(v[u], f);
                // a thread visits its columns in increasing order, so a vector changes its best only with
                // a larger value (at its first column holding the vector's max) or with the thread's first
                // NaN; the vector's NaN-propagating max shows either
                const int c = (int)(c0 + u * step);
                float m = f[0];
#pragma unroll
                for (int e = 1; e < kV; ++e) m = max_nan(m, f[e]);
                if (m != m) {
                    if (best.v == best.v) {
                        int j = 0;
#pragma unroll
                        for (int e = kV - 1; e >= 0; --e) j = (f[e] != f[e]) ? e : j;
                        best.v = m;
                        best.i = c + j;
                    }
                } else if (m > best.v || best.i == INT_MAX) {
                    int j = 0;
#pragma unroll
                    for (int e = kV - 1; e >= 0; --e) j = (f[e] == m) ? e : j;
                    best.v = m;
                    best.i = c + j;
                }
            }
        }
        for (int64_t c = hiv + threadIdx.x; c < hi; c += blockDim.x) best.take(Elem<T>::to_float(row[c]), (int)c);
    } else {
        for (int64_t c = lo + threadIdx.x; c < hi; c += blockDim.x) best.take(Elem<T>::to_float(row[c]), (int)c);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
        best.take(ov, oi);
    }
    // slot (r, s, warp); 0 (below every key) when the warp saw no column
    if ((threadIdx.x & 31) == 0)
        slots[(r * gridDim.x + s) * (blockDim.x >> 5) + (threadIdx.x >> 5)] =
            best.i != INT_MAX ? argmax_key(best.v, best.i) : 0ull;
}

__global__ void __launch_bounds__(256) argmax_keys_kernel(const unsigned long long* __restrict__ slots,
                                                          int64_t* __restrict__ out, int64_t rows, int per_row) {
    griddep_wait();  // the scan has ended and its slots are visible
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    for (int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows;
         r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
        unsigned long long key = 0ull;
        for (int k = lane; k < per_row; k += 32) key = max(key, slots[r * per_row + k]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
        if (lane == 0) out[r] = (int64_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
    }
}

// Column slices per row: 8192 columns (four 16-byte loads in flight per thread
// of 256 for 16-bit logits), narrower (down to 2048) when that leaves fewer than
// two CTAs per SM; a multiple of 8 columns each.
static void argmax_plan(int64_t rows, int64_t cols, int sms, int* splits, int64_t* per) {
    const int64_t by_width = (cols + 8191) / 8192;
    const int64_t want = std::max<int64_t>(by_width, std::min<int64_t>((2 * (int64_t)sms + rows - 1) / rows,
                                                                       (cols + 2047) / 2048));
    int64_t p = (cols + want - 1) / want;
    p = (p + 7) / 8 * 8;
    *per = std::max<int64_t>(p, 8);
    *splits = (int)((cols + *per - 1) / *per);
}

// one 64-bit key slot per (row, slice, warp of 8)
static int64_t argmax_workspace_bytes(int64_t rows, int64_t cols, int sms) {
    int splits;
    int64_t per;
    argmax_plan(rows, cols, sms, &splits, &per);
    return (rows * splits * 8 * 8 + 255) / 256 * 256;
}

template <typename T>
static cudaError_t launch_argmax_typed(const void* x, int64_t rows, int64_t cols, int64_t stride, void* ws,
                                       int64_t* out, int sms, cudaStream_t s) {
    int splits;
    int64_t per;
    argmax_plan(rows, cols, sms, &splits, &per);
    unsigned long long* slots = static_cast<unsigned long long*>(ws);
    const T* xt = static_cast<const T*>(x);
    const bool vec = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (stride * (int64_t)sizeof(T)) % 16 == 0;
    const dim3 grid((unsigned)splits, (unsigned)rows);
    cudaError_t err = vec ? launch_chained(argmax_rows_kernel<T, true>, grid, dim3(256), 0, s, xt, cols, stride, per,
                                           slots)
                          : launch_chained(argmax_rows_kernel<T, false>, grid, dim3(256), 0, s, xt, cols, stride, per,
                                           slots);
    if (err != cudaSuccess) return err;
    const unsigned blocks = (unsigned)std::min<int64_t>((rows + 7) / 8, (int64_t)sms * 4);  // 8 rows (warps) per CTA
    return launch_chained(argmax_keys_kernel, dim3(blocks), dim3(256), 0, s, slots, out, rows, splits * 8);
}

static cudaError_t launch_argmax(int dtype, const void* x, int64_t rows, int64_t cols, int64_t stride, void* ws,
                                 int64_t* out, int sms, cudaStream_t s) {
    if (dtype == MINIKV_F32) return launch_argmax_typed<float>(x, rows, cols, stride, ws, out, sms, s);
    if (dtype == MINIKV_F16) return launch_argmax_typed<__half>(x, rows, cols, stride, ws, out, sms, s);
    return launch_argmax_typed<__nv_bfloat16>(x, rows, cols, stride, ws, out, sms, s);
}

// ---------------------------------------------------------------- launchers
template <typename T>
static cudaError_t launch_rms_norm_typed(const void* x, const void* residual, const void* weight, void* out,
                                        void* sum_out, int64_t rows, int hidden, float eps, cudaStream_t s) {
    const int vecs = hidden / 8;
    int threads = std::min(256, ((vecs + 31) / 32) * 32);
    const int per = (vecs + threads - 1) / threads;
    const T* xt = static_cast<const T*>(x);
    const T* rt = static_cast<const T*>(residual);
    const T* wt = static_cast<const T*>(weight);
    T* ot = static_cast<T*>(out);
    T* st = static_cast<T*>(sum_out);
    const dim3 grid((unsigned)rows);
    if (per <= 1) return launch_chained(rms_norm_kernel<T, 1>, grid, dim3(threads), 0, s, xt, rt, wt, ot, st, hidden, eps);
    if (per <= 2) return launch_chained(rms_norm_kernel<T, 2>, grid, dim3(threads), 0, s, xt, rt, wt, ot, st, hidden, eps);
    return launch_chained(rms_norm_kernel<T, 4>, grid, dim3(threads), 0, s, xt, rt, wt, ot, st, hidden, eps);
}

static cudaError_t launch_rms_norm(int dtype, const void* x, const void* residual, const void* weight, void* out,
                                   void* sum_out, int64_t rows, int hidden, float eps, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    if (dtype == MINIKV_BF16)
        return launch_rms_norm_typed<__nv_bfloat16>(x, residual, weight, out, sum_out, rows, hidden, eps, s);
    return launch_rms_norm_typed<__half>(x, residual, weight, out, sum_out, rows, hidden, eps, s);
}

static cudaError_t launch_silu_mul(int dtype, const void* gate_up, void* out, int64_t rows, int64_t inter,
                                   int sms, cudaStream_t s) {
    const int64_t total = rows * (inter / 8);
    if (total <= 0) return cudaSuccess;
    int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8);
    if (dtype == MINIKV_BF16)
        return launch_chained(silu_mul_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, s,
                              static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), rows,
                              inter);
    return launch_chained(silu_mul_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, s,
                          static_cast<const __half*>(gate_up), static_cast<__half*>(out), rows, inter);
}

template <typename T>
static cudaError_t launch_qk_rope_typed(const QkRopeParams& p, int head_dim, unsigned blocks, cudaStream_t s) {
    switch (head_dim) {
        case 64: return launch_chained(qk_rope_append_kernel<T, 64>, dim3(blocks), dim3(256), 0, s, p);
        case 128: return launch_chained(qk_rope_append_kernel<T, 128>, dim3(blocks), dim3(256), 0, s, p);
        default: return launch_chained(qk_rope_append_kernel<T, 256>, dim3(blocks), dim3(256), 0, s, p);
    }
}

static cudaError_t launch_qk_rope_append(int dtype, const QkRopeParams& p, int head_dim, int sms, cudaStream_t s) {
    const int64_t jobs = p.batch * (p.q_heads + p.kv_heads);
    if (jobs <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((jobs + 7) / 8, (int64_t)sms * 8);
    if (dtype == MINIKV_BF16) return launch_qk_rope_typed<__nv_bfloat16>(p, head_dim, (unsigned)blocks, s);
    return launch_qk_rope_typed<__half>(p, head_dim, (unsigned)blocks, s);
}

}  // namespace minikv
