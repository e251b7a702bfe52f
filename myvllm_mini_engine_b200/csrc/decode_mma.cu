// Tensor-core consumer for the split-KV decode (fp16 / bf16).
//
// Same work decomposition, producer protocol, records and merge as
// paged_decode_split_kernel (decode.cu); only the per-tile math differs.  A
// consumer warp owns one kv head and up to 16 of its query heads and runs the
// tile on the tensor cores with mma.sync m16n8k16 (fp32 accumulate):
//   S[16 heads x 8 tokens]  = Q[16 x 16 dims] . K^T      (K rows via ldmatrix)
//   O[16 heads x D]        += P[16 x 16 tokens] . V      (V rows via ldmatrix.trans)
// The GQA heads of one kv head form the M rows, so every K/V byte staged in
// shared memory is read once per kv head.  Softmax runs on the S fragments in
// registers (row max / sum across the 4-lane quad); P is rounded to the input
// type for the PV product, as in FlashAttention.  Shared-memory token rows are
// padded by 16 bytes (row stride / 16 is odd) so ldmatrix is bank-conflict
// free; the producer therefore copies each token row with its own bulk copy
// and zero-fills the V rows of masked tokens (the MMA multiplies them by P=0,
// which must not meet a NaN bit pattern left in shared memory).
#include "common.cuh"

namespace minikv {

constexpr int kMmaHeads = 16;  // query heads per consumer warp (M rows of the MMA)

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
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

template <typename T, int D>
__global__ void __launch_bounds__(kDecodeThreads, 1) paged_decode_mma_kernel(const DecodeParams p) {
    static_assert(D % 16 == 0, "head_dim must be a multiple of 16");
    constexpr int KSTEPS = D / 16;  // k-steps of the QK product
    constexpr int NTILES = D / 8;   // n-tiles of the PV product
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int warp_sums[kDecodeThreads / 32];

    const int TT = p.tile_tokens, NS = p.stages, stride = p.row_bytes;
    const int stage_bytes = 2 * TT * stride;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * stage_bytes);
    uint64_t* empty = full + NS;
    uint64_t* masks = empty + NS;
    int* prefix = reinterpret_cast<int*>(masks + NS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int B = p.batch;
    const int64_t cap = (int64_t)p.table_width * p.block_size;

    tile_prefix(p.lens, B, cap, TT, prefix, warp_sums);
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init_fence();
    }
    if (blockIdx.x == 0 && blockIdx.y == 0)
        for (int i = tid; i <= B; i += blockDim.x) p.prefix_out[i] = prefix[i];
    __syncthreads();

    const int total = prefix[B];
    const int G = gridDim.x, c = blockIdx.x;
    const int tile_lo = (int)((int64_t)c * total / G), tile_hi = (int)((int64_t)(c + 1) * total / G);
    if (tile_lo >= tile_hi) return;

    const int cph = p.chunks_per_head;  // chunks of kMmaHeads query heads per kv head
    int h0, nh, kvh, chunk;
    bool active;
    if (cph >= kConsumerWarps) {
        h0 = blockIdx.y / p.chunk_groups;
        nh = 1;
        kvh = h0;
        chunk = (blockIdx.y % p.chunk_groups) * kConsumerWarps + warp;
        active = chunk < cph;
    } else {
        h0 = blockIdx.y * p.heads_per_cta;
        nh = min(p.heads_per_cta, p.kv_heads - h0);
        kvh = h0 + warp / cph;
        chunk = warp % cph;
        active = warp < nh * cph;
    }
    constexpr int esize = 2;
    const int copy_row = nh * D * esize;
    const int cache_row = p.kv_heads * D * esize;
    int b = 0;
    {
        int lo = 0, hi = B - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (prefix[mid] <= tile_lo) lo = mid; else hi = mid - 1;
        }
        b = lo;
    }

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        const uint64_t policy = policy_evict_first();
        const unsigned char* kbase = static_cast<const unsigned char*>(p.kc) + (size_t)h0 * D * esize;
        const unsigned char* vbase = static_cast<const unsigned char*>(p.vc) + (size_t)h0 * D * esize;
        int gt = 0;
        for (int t = tile_lo; t < tile_hi;) {
            while (b + 1 < B && prefix[b + 1] <= t) ++b;
            const int seg_hi = min(tile_hi, prefix[b + 1]);
            const int64_t len = p.lens[b];
            const int64_t* table = p.tables + (p.table_rows ? p.table_rows[b] : (int64_t)b) * p.table_width;
            for (int k = t - prefix[b]; k < seg_hi - prefix[b]; ++k, ++gt) {
                const int slot = gt % NS;
                if (gt >= NS) mbar_wait(&empty[slot], ((gt / NS) - 1) & 1);
                const int64_t t0 = (int64_t)k * TT;
                const int n = (int)min((int64_t)TT, len - t0);
                int64_t rows[2];
                bool ok[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int j = lane + 32 * h;
                    ok[h] = false;
                    rows[h] = 0;
                    if (j < n) {
                        const int64_t pos = t0 + j;
                        const int64_t page = table[pos / p.block_size];
                        ok[h] = page >= 0 && page < p.num_blocks;
                        rows[h] = page * p.block_size + pos % p.block_size;
                    }
                }
                const uint64_t mask = (uint64_t)__ballot_sync(0xffffffffu, ok[0]) |
                                      ((uint64_t)__ballot_sync(0xffffffffu, ok[1]) << 32);
                unsigned char* kdst = smem + slot * stage_bytes;
                unsigned char* vdst = kdst + TT * stride;
                // Masked V rows must hold finite values: zero them (generic stores,
                // ordered before the consumers' reads by the arrive below).
                const uint64_t tile_bits = (TT == 64) ? ~0ull : ((1ull << TT) - 1);
                uint64_t holes = ~mask & tile_bits;
                while (holes) {
                    const int j = __ffsll((long long)holes) - 1;
                    holes &= holes - 1;
                    uint4* row = reinterpret_cast<uint4*>(vdst + j * stride);
                    for (int v = lane; v < copy_row / 16; v += 32) row[v] = make_uint4(0, 0, 0, 0);
                }
                __syncwarp();
                if (lane == 0) {
                    masks[slot] = mask;
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)(__popcll(mask) * copy_row * 2));
                }
                __syncwarp();
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int j = lane + 32 * h;
                    if (!ok[h]) continue;
                    bulk_load(kdst + j * stride, kbase + rows[h] * cache_row, copy_row, &full[slot], policy);
                    bulk_load(vdst + j * stride, vbase + rows[h] * cache_row, copy_row, &full[slot], policy);
                }
            }
            t = seg_hi;
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    using Mma = MmaType<T>;
    const int g = lane >> 2, q4 = lane & 3;
    const int item_heads = min(kMmaHeads, p.group - chunk * kMmaHeads);
    const int local_head = kvh - h0;
    uint32_t qa[KSTEPS][4];   // Q as the A operand, rows = query heads
    float o[NTILES][4];       // O accumulators: rows g and g+8, dims 8*nd + 2*q4 (+1)
    float m[2], l[2];         // running max (log2 domain) / partial sum of rows g, g+8
    int gt = 0;
    const uint32_t smem_base = smem_addr(smem);
    // ldmatrix lane addressing (see the fragment layout of m16n8k16)
    const int ld_row = lane & 7, ld_mat = lane >> 3;
    for (int t = tile_lo; t < tile_hi;) {
        while (b + 1 < B && prefix[b + 1] <= t) ++b;
        const int seg_hi = min(tile_hi, prefix[b + 1]);
        const int64_t len = p.lens[b];
        if (active) {
            const T* qbase = static_cast<const T*>(p.q) + ((int64_t)b * p.q_heads + kvh * p.group + chunk * kMmaHeads) * D;
            const bool row_lo = g < item_heads, row_hi = g + 8 < item_heads;
#pragma unroll
            for (int kk = 0; kk < KSTEPS; ++kk) {
                const int d0 = 16 * kk + 2 * q4;
                qa[kk][0] = row_lo ? *reinterpret_cast<const uint32_t*>(qbase + g * D + d0) : 0u;
                qa[kk][1] = row_hi ? *reinterpret_cast<const uint32_t*>(qbase + (g + 8) * D + d0) : 0u;
                qa[kk][2] = row_lo ? *reinterpret_cast<const uint32_t*>(qbase + g * D + d0 + 8) : 0u;
                qa[kk][3] = row_hi ? *reinterpret_cast<const uint32_t*>(qbase + (g + 8) * D + d0 + 8) : 0u;
            }
#pragma unroll
            for (int nd = 0; nd < NTILES; ++nd)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[nd][e] = 0.f;
            m[0] = m[1] = -INFINITY;
            l[0] = l[1] = 0.f;
        }
        for (int k = t - prefix[b]; k < seg_hi - prefix[b]; ++k, ++gt) {
            const int slot = gt % NS;
            mbar_wait(&full[slot], (gt / NS) & 1);
            if (active) {
                const uint64_t mask = masks[slot];
                const int n = (int)min((int64_t)TT, len - (int64_t)k * TT);
                const uint32_t ks = smem_base + slot * stage_bytes + local_head * D * esize;
                const uint32_t vs = ks + TT * stride;
                for (int sub = 0; sub < TT; sub += 16) {
                    // ---- S = Q K^T for 16 tokens (two n-tiles of 8)
                    float s[2][4];
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                        for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
                        const uint32_t krow = ks + (sub + nt * 8 + ld_row) * stride;
#pragma unroll
                        for (int kk = 0; kk + 1 < KSTEPS; kk += 2) {
                            uint32_t r[4];
                            ldsm_x4(krow + (16 * kk + 8 * ld_mat) * esize, r);
                            Mma::mma(s[nt], qa[kk], r[0], r[1]);
                            Mma::mma(s[nt], qa[kk + 1], r[2], r[3]);
                        }
                        if (KSTEPS & 1) {
                            uint32_t r[2];
                            ldsm_x2(krow + (16 * (KSTEPS - 1) + 8 * (ld_mat & 1)) * esize, r);
                            Mma::mma(s[nt], qa[KSTEPS - 1], r[0], r[1]);
                        }
                    }
                    // ---- mask, scale, online softmax on rows g (e = 0,1) and g+8 (e = 2,3)
                    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int j = sub + nt * 8 + 2 * q4 + (e & 1);
                            const bool ok = j < n && ((mask >> j) & 1ull);
                            s[nt][e] = ok ? s[nt][e] * p.scale_log2 : -INFINITY;
                            mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
                        }
                    float alpha[2];
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                        const float mn = fmaxf(m[r], mx[r]);
                        alpha[r] = (mn == -INFINITY) ? 1.f : exp2f(m[r] - mn);
                        m[r] = mn;
                    }
                    uint32_t pa[4];
                    float psum[2] = {0.f, 0.f};
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        float pv[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float mr = m[e >> 1];
                            pv[e] = (mr == -INFINITY) ? 0.f : exp2f(s[nt][e] - mr);
                            psum[e >> 1] += pv[e];
                        }
                        pa[2 * nt] = Elem<T>::pack(pv[0], pv[1]);
                        pa[2 * nt + 1] = Elem<T>::pack(pv[2], pv[3]);
                    }
                    l[0] = l[0] * alpha[0] + psum[0];
                    l[1] = l[1] * alpha[1] + psum[1];
                    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
                        for (int nd = 0; nd < NTILES; ++nd) {
                            o[nd][0] *= alpha[0];
                            o[nd][1] *= alpha[0];
                            o[nd][2] *= alpha[1];
                            o[nd][3] *= alpha[1];
                        }
                    }
                    // ---- O += P V: A = P (tokens 0-7 | 8-15 from the two S n-tiles)
                    const uint32_t afrag[4] = {pa[0], pa[1], pa[2], pa[3]};
                    const uint32_t vrow = vs + (sub + ld_row + 8 * (ld_mat & 1)) * stride;
#pragma unroll
                    for (int nd = 0; nd < NTILES; nd += 2) {
                        uint32_t r[4];
                        ldsm_x4_trans(vrow + (8 * (nd + (ld_mat >> 1))) * esize, r);
                        Mma::mma(o[nd], afrag, r[0], r[1]);
                        Mma::mma(o[nd + 1], afrag, r[2], r[3]);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (active) {
            const bool final_row = cta_of_tile(prefix[b], G, total) == cta_of_tile(prefix[b + 1] - 1, G, total);
            const int record = b + c;
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float L = l[r];
                L += __shfl_xor_sync(0xffffffffu, L, 1);
                L += __shfl_xor_sync(0xffffffffu, L, 2);
                const int row = g + 8 * r;
                if (row >= item_heads) continue;
                const int qh = kvh * p.group + chunk * kMmaHeads + row;
                const float inv = (L > 0.f) ? 1.f / L : 0.f;
                if (final_row) {
                    T* orow = static_cast<T*>(p.out) + ((int64_t)b * p.q_heads + qh) * D;
#pragma unroll
                    for (int nd = 0; nd < NTILES; ++nd)
                        *reinterpret_cast<uint32_t*>(orow + 8 * nd + 2 * q4) =
                            Elem<T>::pack(o[nd][2 * r] * inv, o[nd][2 * r + 1] * inv);
                } else {
                    float* prow = p.partial + ((int64_t)record * p.q_heads + qh) * D;
#pragma unroll
                    for (int nd = 0; nd < NTILES; ++nd)
                        *reinterpret_cast<float2*>(prow + 8 * nd + 2 * q4) =
                            make_float2(o[nd][2 * r] * inv, o[nd][2 * r + 1] * inv);
                    if (q4 == 0)
                        p.lse[(int64_t)record * p.q_heads + qh] = (L > 0.f) ? m[r] + log2f(L) : -INFINITY;
                }
            }
        }
        t = seg_hi;
    }
}

}  // namespace minikv
