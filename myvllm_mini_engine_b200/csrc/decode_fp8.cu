// FP8 KV pool (E4M3 or E5M2): the quantising slot scatter and the
// tensor-core consumer of the split-KV decode kernel for one-byte K/V rows.
//
// Format.  The pool has the 16-bit pool's shape, [num_blocks, block_size,
// kv_heads, head_dim], one OCP FP8 byte per element (E4M3 or E5M2), with one
// fp32 scale for keys and one for values: stored = fp8_rn_satfinite(x * (1 /
// scale)), read back as stored * scale.  It halves the bytes a decode step
// streams.  The reference has no FP8 pool (it is listed there as future
// work); the write follows its slot-scatter contract
// (mini_engine/kernels/csrc/data.cu:196-206: a slot outside the capacity
// writes nothing).
//
// Decode.  The producer warp and the ticketed merge of decode.cu are reused.
// When one CTA holds every kv head (the usual case: a token's row is then
// hpc * D bytes and consecutive rows of a page are contiguous), rows are
// staged unpadded and the producer issues one bulk copy per run of
// consecutive physical rows, a page or more, instead of one per token: per
// token copies of 1 KB rows held the loop at about half the HBM rate.  The
// consumer converts K and V to fp16 in registers, exactly: an E4M3 K pair with
// one cvt (every E4M3 value is an fp16 normal or zero), an E4M3 V pair with
// integer ops (see Fp8Codec), an E5M2 pair with one byte permute (an E5M2
// byte is the high byte of the fp16 of its value).  It
// then runs the transposed mma.sync scheme of decode_mma.cu in fp16:
//   S^T = K Q^T    with Q rounded to fp16 (saturated at +-65504) once per segment;
//   O^T += V^T P^T with P split into fp16 hi + lo terms.
// The key scale is folded into the softmax scale and the value scale into the
// final normalisation.  A dot product does not depend on the order of its
// terms, so the head dims of the k-steps are permuted: lane q4 of k-step kk
// covers dims q4*D/4 + 4kk .. +3, so a lane's K bytes of a token are one
// contiguous D/4-byte run (vector loads), and Q is permuted the same way.
// For V^T (the A operand, dims as rows), a lane loads dims g*D/8 .. +D/8 of
// each of its 4 tokens and pairs the tokens with byte permutes; word w of
// that run feeds m-tiles 2w (rows g, g+8 = dims g*D/8 + 4w + 0, 1) and 2w + 1
// (dims + 2, 3).  On unpadded rows, K reads are conflict-free (odd rows read
// their two 16-byte halves in swapped order) and V reads meet 4-way bank
// conflicts.
#include <cuda_fp8.h>

#include "common.cuh"

namespace minikv {

// Two e4m3 values (low byte first) as an f16x2 (low half first).
__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t pair) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(pair & 0xffffu), __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

__device__ __forceinline__ uint32_t byte_perm(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// NB bytes (a multiple of 4) at p as 32-bit words, in the widest vectors the
// alignment (ALIGN, a power of two >= 4) allows.
template <int NB, int ALIGN>
__device__ __forceinline__ void load_words(const unsigned char* p, uint32_t* w) {
    if constexpr (ALIGN >= 16 && NB % 16 == 0) {
#pragma unroll
        for (int i = 0; i < NB / 16; ++i) {
            const uint4 v = *reinterpret_cast<const uint4*>(p + 16 * i);
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
    } else if constexpr (ALIGN >= 8 && NB % 8 == 0) {
#pragma unroll
        for (int i = 0; i < NB / 8; ++i) {
            const uint2 v = *reinterpret_cast<const uint2*>(p + 8 * i);
            w[2 * i] = v.x; w[2 * i + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < NB / 4; ++i) w[i] = *reinterpret_cast<const uint32_t*>(p + 4 * i);
    }
}

constexpr int pow2_align(int bytes) { return (bytes % 16 == 0) ? 16 : (bytes % 8 == 0) ? 8 : 4; }

// Pairs of fp8 codes to f16x2 for the two formats.  E4M3: the hardware
// conversion (exact).  E5M2: an E5M2 byte is the high byte of the fp16 of the
// same value, so a byte permute is the conversion (exact, ALU only).
//
// For V, E4M3 uses integer ops instead, so that K's conversions and V's run on
// two pipes (XU and ALU): a code s.eeee.mmm placed as fp16 bits
// s.0eeee.mmm0000000 is the fp16 of its value times 2^-8, for normals and
// subnormals alike (fp16 has 8 more exponent bias and room for every E4M3
// subnormal).  vlo/vhi return that; kVScale is the factor the output is
// multiplied back by.
__device__ __forceinline__ uint32_t e4m3x2_to_h2_scaled(uint32_t spread) {
    // spread = code0 << 8 | code1 << 24: shift the magnitudes into place, then move
    // the sign from bit 14 (30) to 15 (31) by adding the bit to itself
    const uint32_t t = spread >> 1;
    return t + (t & 0x40004000u);
}
template <bool E5M2> struct Fp8Codec;
template <> struct Fp8Codec<false> {
    __device__ static __forceinline__ uint32_t lo(uint32_t w) { return e4m3x2_to_h2(w); }        // bytes 0, 1
    __device__ static __forceinline__ uint32_t hi(uint32_t w) { return e4m3x2_to_h2(w >> 16); }  // bytes 2, 3
    __device__ static __forceinline__ uint32_t vlo(uint32_t w) { return e4m3x2_to_h2_scaled(byte_perm(w, 0u, 0x1404u)); }
    __device__ static __forceinline__ uint32_t vhi(uint32_t w) { return e4m3x2_to_h2_scaled(byte_perm(w, 0u, 0x3424u)); }
    static constexpr float kVScale = 256.f;
};
template <> struct Fp8Codec<true> {
    __device__ static __forceinline__ uint32_t lo(uint32_t w) { return byte_perm(w, 0u, 0x1404u); }
    __device__ static __forceinline__ uint32_t hi(uint32_t w) { return byte_perm(w, 0u, 0x3424u); }
    __device__ static __forceinline__ uint32_t vlo(uint32_t w) { return lo(w); }
    __device__ static __forceinline__ uint32_t vhi(uint32_t w) { return hi(w); }
    static constexpr float kVScale = 1.f;
};

// fp16 pair of two floats, saturated to the finite fp16 range.
__device__ __forceinline__ uint32_t h2_sat(float a, float b) {
    a = fminf(fmaxf(a, -65504.f), 65504.f);
    b = fminf(fmaxf(b, -65504.f), 65504.f);
    return Elem<__half>::pack(a, b);
}

template <typename T, int D, bool E5M2>
struct Fp8MmaConsumer {
    static_assert(D % 32 == 0, "the fp8 pool needs head_dim % 32 == 0");
    static constexpr int KSTEPS = D / 16;  // k-steps of S^T = K Q^T
    static constexpr int GROUPS = D / 32;  // V words per token and lane (two m-tiles each)
    static constexpr int KB = D / 4;       // K bytes of a token per lane
    static constexpr int VB = D / 8;       // V bytes of a token per lane
    static constexpr int kKvBytes = 1;     // bytes per cached element
    static constexpr bool kPairCapable = false;  // rows staged unpadded (runs) or padded, one per stride
    static constexpr bool kE5M2 = E5M2;          // the pool's byte format (the fused append quantises to it)
    using Mma = MmaType<__half>;
    using Codec = Fp8Codec<E5M2>;

    uint32_t qb[KSTEPS][2];  // Q^T (fp16): head g, dims q4*D/4 + 4kk + {0,1} and + {2,3}
    float o[2 * GROUPS][4];  // O^T: m-tile 2w + i, row g -> dim g*D/8 + 4w + 2i, row g + 8 -> + 1
    float m[2], l[2];
    int g, q4;

    __device__ void setup(int lane) {
        g = lane >> 2;
        q4 = lane & 3;
    }

    __device__ void begin(const T* qrows, int item_heads) {
        const bool valid = g < item_heads;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
            float f[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) f[i] = valid ? Elem<T>::to_float(qrows[g * D + q4 * KB + 4 * kk + i]) : 0.f;
            qb[kk][0] = h2_sat(f[0], f[1]);
            qb[kk][1] = h2_sat(f[2], f[3]);
        }
#pragma unroll
        for (int mt = 0; mt < 2 * GROUPS; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
    }

    // A lane's K run of one token (KB bytes).  Runs of 32 bytes are read as two
    // 16-byte halves, odd rows g first the upper one: rows g and g + 1 of a
    // quarter-warp then hit different banks when rows are unpadded.
    __device__ __forceinline__ void load_k_run(const unsigned char* p, uint32_t* w) const {
        if constexpr (KB == 32) {
            const int first = (g & 1) ? 16 : 0;
            const uint4 a = *reinterpret_cast<const uint4*>(p + first);
            const uint4 b = *reinterpret_cast<const uint4*>(p + (16 - first));
            const uint4 lo = (g & 1) ? b : a, hi = (g & 1) ? a : b;
            w[0] = lo.x; w[1] = lo.y; w[2] = lo.z; w[3] = lo.w;
            w[4] = hi.x; w[5] = hi.y; w[6] = hi.z; w[7] = hi.w;
        } else {
            load_words<KB, pow2_align(KB)>(p, w);
        }
    }

    __device__ void tile(const unsigned char* kptr, const unsigned char* vptr, int stride, int TT, int n,
                         uint64_t mask, float scale_log2, bool = false) {
        // Two 16-token slices per step where the tile allows: their K loads,
        // conversions and MMAs are independent (ILP for a warp that is alone with
        // one other on its scheduler), and the online-softmax max, rescale and
        // exp2 of alpha are paid once per 32 tokens.
        int sub = 0;
        for (; sub + 32 <= TT; sub += 32) step<2>(kptr, vptr, stride, sub, n, mask, scale_log2);
        for (; sub < TT; sub += 16) step<1>(kptr, vptr, stride, sub, n, mask, scale_log2);
    }

    template <int NS>
    __device__ __forceinline__ void step(const unsigned char* kptr, const unsigned char* vptr, int stride, int sub,
                                         int n, uint64_t mask, float scale_log2) {
        // ---- S^T = K Q^T: lane (g, q4) reads dims q4*D/4 .. +D/4 of tokens g and g + 8 of each slice
        float s[NS][4], s2[NS][4];
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            uint32_t kw0[KSTEPS], kw1[KSTEPS];
            load_k_run(kptr + (sub + 16 * i + g) * stride + q4 * KB, kw0);
            load_k_run(kptr + (sub + 16 * i + g + 8) * stride + q4 * KB, kw1);
#pragma unroll
            for (int e = 0; e < 4; ++e) s[i][e] = s2[i][e] = 0.f;
#pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) {
                uint32_t a[4];
                a[0] = Codec::lo(kw0[kk]);
                a[1] = Codec::lo(kw1[kk]);
                a[2] = Codec::hi(kw0[kk]);
                a[3] = Codec::hi(kw1[kk]);
                Mma::mma((kk & 1) ? s2[i] : s[i], a, qb[kk][0], qb[kk][1]);
            }
        }
        // V words of every slice, loaded before the softmax so their latency overlaps it:
        // lane (g, q4) reads dims g*D/8 .. +D/8 of tokens 2q4, 2q4+1, 2q4+8, 2q4+9
        uint32_t vw[NS][4][GROUPS];
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            const unsigned char* v0 = vptr + (sub + 16 * i + 2 * q4) * stride + g * VB;
            load_words<VB, pow2_align(VB)>(v0, vw[i][0]);
            load_words<VB, pow2_align(VB)>(v0 + stride, vw[i][1]);
            load_words<VB, pow2_align(VB)>(v0 + 8 * stride, vw[i][2]);
            load_words<VB, pow2_align(VB)>(v0 + 9 * stride, vw[i][3]);
        }
        // ---- mask and scale (as decode_mma.cu; the key scale is in scale_log2)
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            const int j0 = sub + 16 * i + g, j1 = j0 + 8;
            const bool ok0 = j0 < n && ((mask >> j0) & 1ull), ok1 = j1 < n && ((mask >> j1) & 1ull);
            s[i][0] = ok0 ? (s[i][0] + s2[i][0]) * scale_log2 : -INFINITY;
            s[i][1] = ok0 ? (s[i][1] + s2[i][1]) * scale_log2 : -INFINITY;
            s[i][2] = ok1 ? (s[i][2] + s2[i][2]) * scale_log2 : -INFINITY;
            s[i][3] = ok1 ? (s[i][3] + s2[i][3]) * scale_log2 : -INFINITY;
        }
        float alpha[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float mx = fmaxf(s[0][h], s[0][h + 2]);
#pragma unroll
            for (int i = 1; i < NS; ++i) mx = fmaxf(mx, fmaxf(s[i][h], s[i][h + 2]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(m[h], mx);
            alpha[h] = (mn == -INFINITY) ? 1.f : exp2f(m[h] - mn);
            m[h] = mn;
        }
        float pv[NS][4];
#pragma unroll
        for (int i = 0; i < NS; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) pv[i][e] = (m[e & 1] == -INFINITY) ? 0.f : exp2f(s[i][e] - m[e & 1]);
        float add0 = 0.f, add1 = 0.f;
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            add0 += pv[i][0] + pv[i][2];
            add1 += pv[i][1] + pv[i][3];
        }
        l[0] = l[0] * alpha[0] + add0;
        l[1] = l[1] * alpha[1] + add1;
        if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
            for (int mt = 0; mt < 2 * GROUPS; ++mt) {
                o[mt][0] *= alpha[0];
                o[mt][1] *= alpha[1];
                o[mt][2] *= alpha[0];
                o[mt][3] *= alpha[1];
            }
        }
#pragma unroll
        for (int i = 0; i < NS; ++i) {
            // ---- P = P_hi + P_lo in fp16, moved into the B layout (as decode_mma.cu)
            const uint32_t h01 = Elem<__half>::pack(pv[i][0], pv[i][1]);
            const uint32_t h23 = Elem<__half>::pack(pv[i][2], pv[i][3]);
            float rest[4];
            {
                float back[4];
                Elem<__half>::unpack(h01, back);
                Elem<__half>::unpack(h23, back + 2);
#pragma unroll
                for (int e = 0; e < 4; ++e) rest[e] = pv[i][e] - back[e];
            }
            const uint32_t l01 = Elem<__half>::pack(rest[0], rest[1]);
            const uint32_t l23 = Elem<__half>::pack(rest[2], rest[3]);
            const int src0 = (2 * q4) * 4 + (g >> 1), src1 = src0 + 4;
            const bool odd = g & 1;
            const uint32_t b0 = pick_halves(__shfl_sync(0xffffffffu, h01, src0), __shfl_sync(0xffffffffu, h01, src1), odd);
            const uint32_t b1 = pick_halves(__shfl_sync(0xffffffffu, h23, src0), __shfl_sync(0xffffffffu, h23, src1), odd);
            const uint32_t c0 = pick_halves(__shfl_sync(0xffffffffu, l01, src0), __shfl_sync(0xffffffffu, l01, src1), odd);
            const uint32_t c1 = pick_halves(__shfl_sync(0xffffffffu, l23, src0), __shfl_sync(0xffffffffu, l23, src1), odd);
            // ---- O^T += V^T P^T
#pragma unroll
            for (int u = 0; u < GROUPS; ++u) {
                const uint32_t w0 = vw[i][0][u], w1 = vw[i][1][u], w2 = vw[i][2][u], w3 = vw[i][3][u];
                // byte i of word u is dim g*D/8 + 4u + i; pair the two tokens of each k slot
                const uint32_t x01 = byte_perm(w0, w1, 0x5140u), x23 = byte_perm(w2, w3, 0x5140u);  // dims +0, +1
                const uint32_t y01 = byte_perm(w0, w1, 0x7362u), y23 = byte_perm(w2, w3, 0x7362u);  // dims +2, +3
                uint32_t a[4];
                a[0] = Codec::vlo(x01);
                a[1] = Codec::vhi(x01);
                a[2] = Codec::vlo(x23);
                a[3] = Codec::vhi(x23);
                Mma::mma(o[2 * u], a, c0, c1);
                Mma::mma(o[2 * u], a, b0, b1);
                a[0] = Codec::vlo(y01);
                a[1] = Codec::vhi(y01);
                a[2] = Codec::vlo(y23);
                a[3] = Codec::vhi(y23);
                Mma::mma(o[2 * u + 1], a, c0, c1);
                Mma::mma(o[2 * u + 1], a, b0, b1);
            }
        }
    }

    __device__ void finish(const DecodeParams& p, int b, int qh0, int item_heads, bool final_row, int64_t record) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float L = l[h];
            L += __shfl_xor_sync(0xffffffffu, L, 4);
            L += __shfl_xor_sync(0xffffffffu, L, 8);
            L += __shfl_xor_sync(0xffffffffu, L, 16);
            const int head = 2 * q4 + h;
            if (head >= item_heads) continue;
            const int qh = qh0 + head;
            const float inv = (L > 0.f) ? p.out_scale * Codec::kVScale / L : 0.f;  // the value scale folded in
            if (final_row) {
                T* orow = static_cast<T*>(p.out) + ((int64_t)b * p.q_heads + qh) * D;
#pragma unroll
                for (int u = 0; u < GROUPS; ++u) {
                    T* dst = orow + g * VB + 4 * u;
                    dst[0] = Elem<T>::from_float(o[2 * u][h] * inv);
                    dst[1] = Elem<T>::from_float(o[2 * u][h + 2] * inv);
                    dst[2] = Elem<T>::from_float(o[2 * u + 1][h] * inv);
                    dst[3] = Elem<T>::from_float(o[2 * u + 1][h + 2] * inv);
                }
            } else {
                float* prow = p.partial + (record * p.q_heads + qh) * D;
#pragma unroll
                for (int u = 0; u < GROUPS; ++u)
                    *reinterpret_cast<float4*>(prow + g * VB + 4 * u) =
                        make_float4(o[2 * u][h] * inv, o[2 * u][h + 2] * inv, o[2 * u + 1][h] * inv,
                                    o[2 * u + 1][h + 2] * inv);
                if (g == 0) p.lse[record * p.q_heads + qh] = (L > 0.f) ? m[h] + log2f(L) : -INFINITY;
            }
        }
    }
};

// ------------------------------------------------------ quantising scatter
// One warp per token: K and V rows of `row_elems` elements quantised by
// quantize_row_warp (the fused fp8 append of the decode kernel uses the same
// function, so the two write identical bytes).
template <typename T, bool E5M2>
__global__ void __launch_bounds__(256) quantize_slots_kernel(
    unsigned char* __restrict__ kc, unsigned char* __restrict__ vc, const T* __restrict__ k,
    const T* __restrict__ v, const int64_t* __restrict__ slots, int64_t tokens, int64_t capacity,
    int64_t row_elems, int64_t k_stride, int64_t v_stride, float k_inv, float v_inv) {
    griddep_wait();
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < tokens; t += warps) {
        const int64_t slot = slots[t];
        if (slot < 0 || slot >= capacity) continue;  // data.cu:196-206
#pragma unroll
        for (int which = 0; which < 2; ++which) {
            const T* src = which ? v + t * v_stride : k + t * k_stride;
            unsigned char* dst = (which ? vc : kc) + slot * row_elems;
            quantize_row_warp<T, E5M2>(dst, src, (int)row_elems, which ? v_inv : k_inv, lane);
        }
    }
}

template <typename T>
static cudaError_t launch_quantize_slots(void* kc, void* vc, const void* k, const void* v, const int64_t* slots,
                                         int64_t tokens, int64_t capacity, int64_t row_elems, int64_t k_stride,
                                         int64_t v_stride, float k_inv, float v_inv, bool e5m2, cudaStream_t stream) {
    if (tokens <= 0) return cudaSuccess;
    int64_t blocks = (tokens + 7) / 8;
    const int64_t cap = (int64_t)sm_count_for_current_device() * 8;
    if (blocks > cap) blocks = cap;
    return launch_chained(e5m2 ? quantize_slots_kernel<T, true> : quantize_slots_kernel<T, false>,
                          dim3((unsigned)blocks), dim3(256), 0, stream,
                          static_cast<unsigned char*>(kc), static_cast<unsigned char*>(vc),
                          static_cast<const T*>(k), static_cast<const T*>(v), slots, tokens, capacity, row_elems,
                          k_stride, v_stride, k_inv, v_inv);
}

// ------------------------------------------------------------ decode host side
template <typename T, int D, bool E5M2>
static cudaError_t launch_decode_fp8_typed(const DecodeParams& p, const DecodePlan& plan, cudaStream_t stream) {
    auto kernel = paged_decode_kernel<T, D, Fp8MmaConsumer<T, D, E5M2>>;
    static int configured[64] = {0};  // opt-in shared-memory size set per device
    cudaError_t err = ensure_smem_limit(kernel, plan.smem_bytes, configured);
    if (err != cudaSuccess) return err;
    return launch_chained(kernel, dim3(plan.grid, plan.head_groups), dim3(kDecodeThreads), plan.smem_bytes, stream, p);
}

template <typename T, bool E5M2>
static cudaError_t launch_decode_fp8_dim(int D, const DecodeParams& p, const DecodePlan& plan, cudaStream_t stream) {
    switch (D) {
        case 32: return launch_decode_fp8_typed<T, 32, E5M2>(p, plan, stream);
        case 64: return launch_decode_fp8_typed<T, 64, E5M2>(p, plan, stream);
        case 96: return launch_decode_fp8_typed<T, 96, E5M2>(p, plan, stream);
        case 128: return launch_decode_fp8_typed<T, 128, E5M2>(p, plan, stream);
        case 192: return launch_decode_fp8_typed<T, 192, E5M2>(p, plan, stream);
        case 256: return launch_decode_fp8_typed<T, 256, E5M2>(p, plan, stream);
        default: return cudaErrorInvalidValue;
    }
}

template <typename T>
static cudaError_t launch_decode_fp8(bool e5m2, int D, const DecodeParams& p, const DecodePlan& plan,
                                     cudaStream_t stream) {
    return e5m2 ? launch_decode_fp8_dim<T, true>(D, p, plan, stream) : launch_decode_fp8_dim<T, false>(D, p, plan, stream);
}

static bool fp8_head_dim(int64_t d) { return d == 32 || d == 64 || d == 96 || d == 128 || d == 192 || d == 256; }

}  // namespace minikv
