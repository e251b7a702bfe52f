// Tensor-core consumer of the split-KV decode kernel (fp16 / bf16).
//
// A consumer warp owns one kv head and up to 8 of its query heads.  Each
// 16-token slice of a staged tile runs on the tensor cores with mma.sync
// m16n8k16 (fp32 accumulate) in the transposed form, tokens as the M rows and
// the GQA query heads as the N columns:
//   S^T[16 tokens x 8 heads]  = K[16 x 16 dims] . Q^T          (A = K via ldmatrix)
//   O^T[16 dims x 8 heads]   += V^T[16 dims x 16 tokens] . P^T (A = V via ldmatrix.trans)
// so a slice costs D/16 + 2 D/16 MMAs whatever the group size (<= 8), every K/V
// byte staged in shared memory is read once per kv head, and the Q operand
// (16 registers for D=128) and the O accumulators (32) stay small.  Softmax
// runs on the S^T fragments: the max and sum of a head are reductions across
// the 8 lanes that share its column.  P is split into two terms of the input
// type (P_hi + P_lo), each packed and moved into the B-operand layout with
// four shuffles, and both are multiplied into O.  Token rows in
// shared memory are padded (stride / 16 odd), so ldmatrix is bank-conflict
// free; masked tokens' V rows are zero (see the producer).
#include "common.cuh"

namespace minikv {

template <typename T> struct MmaType;
template <> struct MmaType<__half> {
    __device__ static __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct MmaType<__nv_bfloat16> {
    __device__ static __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr) : "memory");
}

// Low or high 16-bit half of x (selected by `high`) into the low half of the
// result, and the same half of y into the high half.
__device__ __forceinline__ uint32_t pick_halves(uint32_t x, uint32_t y, bool high) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(x), "r"(y), "r"(high ? 0x7632u : 0x5410u));
    return r;
}

template <typename T, int D>
struct MmaConsumer {
    static_assert(D % 16 == 0, "head_dim must be a multiple of 16");
    static constexpr int KSTEPS = D / 16;  // k-steps of S^T = K Q^T
    static constexpr int MTILES = D / 16;  // m-tiles (16 dims) of O^T
    static constexpr int esize = 2;
    static constexpr int kKvBytes = 2;  // bytes per cached element
    static constexpr bool kPairCapable = true;  // reads rows staged in pairs (see stage_row_offset)
    using Mma = MmaType<T>;

    uint32_t qb[KSTEPS][2];  // Q^T as the B operand: head g, dims 16kk + 2*q4 (+1) and +8
    float o[MTILES][4];      // O^T: dims 16mt + g (e=0,1) / + g + 8 (e=2,3), heads 2*q4 + (e & 1)
    float m[2], l[2];        // running max (log2 domain) / lane-partial sum of heads 2*q4, 2*q4+1
    int g, q4, ld_row, ld_mat;

    __device__ void setup(int lane) {
        g = lane >> 2;
        q4 = lane & 3;
        ld_row = lane & 7;   // ldmatrix: row of the 8x8 matrix this lane addresses
        ld_mat = lane >> 3;  // ... and which of the four matrices
    }

    __device__ void begin(const T* qrows, int item_heads) {
        const bool valid = g < item_heads;
#pragma unroll
        for (int kk = 0; kk < KSTEPS; ++kk) {
            const int d0 = 16 * kk + 2 * q4;
            qb[kk][0] = valid ? *reinterpret_cast<const uint32_t*>(qrows + g * D + d0) : 0u;
            qb[kk][1] = valid ? *reinterpret_cast<const uint32_t*>(qrows + g * D + d0 + 8) : 0u;
        }
#pragma unroll
        for (int mt = 0; mt < MTILES; ++mt)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[mt][e] = 0.f;
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
    }

    // Rows are padded (`stride` bytes apart) or, with `pair`, staged in pairs (`stride` bytes
    // per pair of tokens, the pair's two rows adjacent).  M row r of a 16-token slice is
    // token r, or with pairs token 2r (r < 8) / 2(r - 8) + 1: even and odd tokens form the
    // two 8-row groups.  Either way the 8 rows one ldmatrix reads are `stride` apart
    // (stride / 16 odd: no bank conflict).  The k index of the P V product follows the
    // same order, so only the token of a row changes, not the MMA data flow.
    __device__ void tile(const unsigned char* kptr, const unsigned char* vptr, int stride, int TT, int n,
                         uint64_t mask, float scale_log2, bool pair = false) {
        const uint32_t ks = smem_addr(kptr), vs = smem_addr(vptr);
        const int row_bytes = (stride - 16) / 2;
        // ldmatrix row addresses: K (A, non-transposed) and V (A of O^T, transposed)
        const int k_off = pair ? ld_row * stride + (ld_mat & 1) * row_bytes : (ld_row + 8 * (ld_mat & 1)) * stride;
        const int v_off = pair ? ld_row * stride + (ld_mat >> 1) * row_bytes : (ld_row + 8 * (ld_mat >> 1)) * stride;
        const int k_dim = 8 * (ld_mat >> 1), v_dim = 8 * (ld_mat & 1);
        const int slice_bytes = pair ? 8 * stride : 16 * stride;
        for (int sub = 0; sub < TT; sub += 16) {
            // ---- S^T = K Q^T, two independent k chains
            float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
            const uint32_t krow = ks + (sub / 16) * slice_bytes + k_off + k_dim * esize;
#pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) {
                uint32_t a[4];
                ldsm_x4(krow + 16 * kk * esize, a);
                Mma::mma((kk & 1) ? s2 : s, a, qb[kk][0], qb[kk][1]);
            }
            // ---- mask and scale: s[0,1] is M row g, s[2,3] row g+8 (tokens sub+g / sub+g+8, or
            // with pairs sub+2g / sub+2g+1); columns heads 2q4, 2q4+1
            const int j0 = pair ? sub + 2 * g : sub + g, j1 = pair ? j0 + 1 : j0 + 8;
            const bool ok0 = j0 < n && ((mask >> j0) & 1ull), ok1 = j1 < n && ((mask >> j1) & 1ull);
            s[0] = ok0 ? (s[0] + s2[0]) * scale_log2 : -INFINITY;
            s[1] = ok0 ? (s[1] + s2[1]) * scale_log2 : -INFINITY;
            s[2] = ok1 ? (s[2] + s2[2]) * scale_log2 : -INFINITY;
            s[3] = ok1 ? (s[3] + s2[3]) * scale_log2 : -INFINITY;
            // ---- online softmax per head column (reduce over the 8 lanes with this q4)
            float alpha[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float mx = fmaxf(s[h], s[h + 2]);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mn = fmaxf(m[h], mx);
                alpha[h] = (mn == -INFINITY) ? 1.f : exp2f(m[h] - mn);
                m[h] = mn;
            }
            float pv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) pv[e] = (m[e & 1] == -INFINITY) ? 0.f : exp2f(s[e] - m[e & 1]);
            l[0] = l[0] * alpha[0] + pv[0] + pv[2];
            l[1] = l[1] * alpha[1] + pv[1] + pv[3];
            if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
                for (int mt = 0; mt < MTILES; ++mt) {
                    o[mt][0] *= alpha[0];
                    o[mt][1] *= alpha[1];
                    o[mt][2] *= alpha[0];
                    o[mt][3] *= alpha[1];
                }
            }
            // ---- P = P_hi + P_lo, both in the input type (P_lo = P - P_hi rounded), so
            // the PV product carries P to ~2^-16 relative, as the reference's fp32
            // probabilities do (fallback.py:59-63), at the cost of one more MMA per m-tile.
            float rest[4];
            const uint32_t h01 = Elem<T>::pack(pv[0], pv[1]);  // token sub+g,   heads 2q4, 2q4+1
            const uint32_t h23 = Elem<T>::pack(pv[2], pv[3]);  // token sub+g+8, heads 2q4, 2q4+1
            {
                float back[4];
                Elem<T>::unpack(h01, back);
                Elem<T>::unpack(h23, back + 2);
#pragma unroll
                for (int e = 0; e < 4; ++e) rest[e] = pv[e] - back[e];
            }
            const uint32_t l01 = Elem<T>::pack(rest[0], rest[1]);
            const uint32_t l23 = Elem<T>::pack(rest[2], rest[3]);
            // ---- P^T into the B layout: lane (g, q4) needs tokens 2q4, 2q4+1 (b0) and
            // 2q4+8, 2q4+9 (b1) of head g; lane (t, h/2) holds tokens t, t+8 of heads h&~1, h|1.
            const int src0 = (2 * q4) * 4 + (g >> 1), src1 = src0 + 4;
            const bool odd = g & 1;
            const uint32_t b0 = pick_halves(__shfl_sync(0xffffffffu, h01, src0), __shfl_sync(0xffffffffu, h01, src1), odd);
            const uint32_t b1 = pick_halves(__shfl_sync(0xffffffffu, h23, src0), __shfl_sync(0xffffffffu, h23, src1), odd);
            const uint32_t c0 = pick_halves(__shfl_sync(0xffffffffu, l01, src0), __shfl_sync(0xffffffffu, l01, src1), odd);
            const uint32_t c1 = pick_halves(__shfl_sync(0xffffffffu, l23, src0), __shfl_sync(0xffffffffu, l23, src1), odd);
            // ---- O^T += V^T P_hi^T + V^T P_lo^T
            const uint32_t vrow = vs + (sub / 16) * slice_bytes + v_off + v_dim * esize;
#pragma unroll
            for (int mt = 0; mt < MTILES; ++mt) {
                uint32_t a[4];
                ldsm_x4_trans(vrow + 16 * mt * esize, a);
                Mma::mma(o[mt], a, c0, c1);
                Mma::mma(o[mt], a, b0, b1);
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
            const float inv = (L > 0.f) ? 1.f / L : 0.f;
            if (final_row) {
                T* orow = static_cast<T*>(p.out) + ((int64_t)b * p.q_heads + qh) * D;
#pragma unroll
                for (int mt = 0; mt < MTILES; ++mt) {
                    orow[16 * mt + g] = Elem<T>::from_float(o[mt][h] * inv);
                    orow[16 * mt + g + 8] = Elem<T>::from_float(o[mt][h + 2] * inv);
                }
            } else {
                float* prow = p.partial + (record * p.q_heads + qh) * D;
#pragma unroll
                for (int mt = 0; mt < MTILES; ++mt) {
                    prow[16 * mt + g] = o[mt][h] * inv;
                    prow[16 * mt + g + 8] = o[mt][h + 2] * inv;
                }
                if (g == 0) p.lse[record * p.q_heads + qh] = (L > 0.f) ? m[h] + log2f(L) : -INFINITY;
            }
        }
    }
};

}  // namespace minikv
