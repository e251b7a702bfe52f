// Split-KV (flash-decoding) paged decode attention for sm_100a.
//
// Work decomposition ("balanced split-KV").  The tokens of every request are
// cut into tiles of TT tokens; the tiles of the whole batch form one list of
// `total` tiles and CTA c of a persistent grid of G CTAs (one per SM) takes
// tiles [c*total/G, (c+1)*total/G).  A CTA therefore streams an equal share of
// the batch's KV bytes whatever the (ragged) lengths are; its range covers one
// or more request *segments*.  A segment that is a whole request writes the
// final output.  Otherwise it writes an fp32 partial (its output normalised by
// its own softmax sum) and its log2-sum-exp, takes a ticket on the request's
// counter, and the CTA holding the last ticket merges the partials
// (exp-weighted by log-sum-exp, as the reference's second pass does,
// mini_engine/kernels/csrc/paged_attention.cu:195-215) -- inside this kernel,
// so there is no second launch.  The grid, the workspace and the record layout
// depend only on (batch, table width, block size, heads, head dim, dtype) and
// the SM count, never on context_lens, so a captured CUDA graph stays valid
// when lengths change (the reference derives its partition count from the
// table width for the same reason, paged_attention.cu:271).
//
// CTA layout: 8 consumer warps + 1 producer warp + 1 ticket warp.  The
// ticket warp takes the merge tickets of the segments that end inside the
// CTA's range (a request boundary mid-range), so the consumers move on to the
// next request as soon as their partial is stored; the segment that ends the
// CTA's range is ticketed (and merged) by the consumers.  The producer first reads
// the physical rows of the next 32 tiles into shared memory with independent
// loads (one page-table lookup per page, all in flight together), then stages
// every tile's K and V rows -- all kv heads of the CTA's head group -- into
// shared memory with 1-D bulk copies (TMA engine), on a ring of `stages`
// buffers guarded by full/empty mbarriers.  Token rows in shared memory are
// padded by 16 bytes.  Each consumer warp owns one kv head and some of its
// query heads (GQA: every KV byte is read from HBM once per step, whatever the
// group size):
//  * fp16/bf16: tensor-core consumer (decode_mma.cu), up to 8 query heads per
//    warp as the N columns of mma.sync m16n8k16 (tokens are the M rows);
//  * fp32: CUDA-core consumer below, two query heads per warp, lane groups
//    with their own online softmax merged at segment end.
//
// Trusted-mode guards of the reference kernel are kept: a page id outside
// [0, num_blocks) masks its tokens (score -inf, paged_attention.cu:72-82); a
// length outside [1, table_width*block_size] yields an all-zero row (:62-64);
// a row with no unmasked token yields zeros (:99, :120).
#include <cuda_fp8.h>

#include "common.cuh"

namespace minikv {

constexpr int kConsumerWarps = 8;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kTicketWarp = kConsumerWarps + 1;
constexpr int kDecodeThreads = (kConsumerWarps + 2) * 32;
constexpr int kCoreHeads = 2;       // query heads per CUDA-core consumer warp
constexpr int kMmaHeads = 8;        // query heads per tensor-core consumer warp (MMA N)
constexpr int kTokensPerGroup = 4;  // CUDA-core: tokens per lane group per sub-chunk
constexpr int kWindowTiles = 32;    // tiles whose rows the producer prefetches at once

struct DecodeParams {
    const void* q;
    const void* kc;
    const void* vc;
    const int64_t* tables;
    const int64_t* lens;
    const int64_t* table_rows;  // table row of request b (nullptr: row b)
    void* out;
    float* partial;             // [records, q_heads, D]
    float* lse;                 // [records, q_heads]   (log2 domain)
    unsigned int* tickets;      // [batch, head groups], zero before the launch; left zero after it
    int batch, q_heads, kv_heads, num_blocks, block_size, table_width;
    int group;            // q_heads / kv_heads
    int heads_per_item;   // query heads per consumer warp
    int chunks_per_head;  // ceil(group / heads_per_item)
    int heads_per_cta;    // kv heads per CTA head group (1 when chunks_per_head >= 8)
    int chunk_groups;     // head groups per kv head (> 1 only when chunks_per_head > 8)
    int tile_tokens;      // TT, multiple of the consumer's sub-chunk, <= 64
    int stages;
    int row_stride;       // shared-memory stride of one token row (padded), or of a pair of rows
    int pair_rows;        // 1: rows staged in pairs (tensor-core consumer, every kv head in the CTA)
    int early_prologue;   // 1: lens/tables predate the previous kernel; read them before griddep_wait
    int coalesce;         // 1: rows unpadded and the CTA holds every kv head: one bulk copy per run of
                          //    consecutive physical rows (fp8 pool only)
    int append;           // 1: fused KV append.  `lens` holds token offsets: request b appends new_k[b] /
                          //    new_v[b] at position lens[b] and attends lens[b] + 1 tokens
    const void* new_k;    // [batch, kv_heads, D] rows appended (append mode)
    const void* new_v;
    float scale_log2;     // log2(e) / sqrt(D) (times the key scale for an fp8 pool)
    float out_scale;      // fp8 pool: the value scale, applied to the output (unused otherwise)
    float k_inv, v_inv;   // fp8 pool with the fused append: 1 / scale, the new rows' quantisation factors
};

// CTA c of G owns tiles [c*total/G, (c+1)*total/G); cta_of_tile(t) inverts it.
__device__ __forceinline__ int cta_of_tile(int t, int G, int total) {
    return (int)((((int64_t)t + 1) * G + total - 1) / total) - 1;
}
__device__ __forceinline__ bool cta_owns_tiles(int cta, int G, int total) {
    // with at least one tile per CTA every CTA owns some (and the 64-bit divisions are skipped)
    return total >= G || ((int64_t)cta * total) / G != ((int64_t)(cta + 1) * total) / G;
}

// One warp quantises a row of `elems` values of T (16 per lane step) into an fp8
// pool row as fp8(x * inv): the fp32 product, then nearest-even with saturation
// to the largest finite code.  Used by the quantising slot scatter and by the
// fused append into an fp8 pool, so both write the same bytes.
template <typename T, bool E5M2>
__device__ __forceinline__ void quantize_row_warp(unsigned char* dst, const T* src, int elems, float inv, int lane) {
    for (int c = lane * 16; c < elems; c += 32 * 16) {
        uint32_t word[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            uint32_t packed = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float x = __fmul_rn(Elem<T>::to_float(src[c + 4 * w + i]), inv);
                packed |= (uint32_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, E5M2 ? __NV_E5M2 : __NV_E4M3) << (8 * i);
            }
            word[w] = packed;
        }
        *reinterpret_cast<uint4*>(dst + c) = make_uint4(word[0], word[1], word[2], word[3]);
    }
}

// Offset of token j's row in a staged tile: rows `stride` apart, or (paired
// staging) pairs of rows `stride` apart, the two rows of a pair adjacent.
__device__ __forceinline__ int stage_row_offset(bool pair, int j, int stride, int row_bytes) {
    return pair ? (j >> 1) * stride + (j & 1) * row_bytes : j * stride;
}

// Consumer-only barrier (the producer warp never joins it).
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32) : "memory");
}

// lens_s[b] = usable length (0 when out of range); prefix[0..B] = exclusive
// prefix of per-request tile counts.  All threads of the CTA take part.  With
// `plus_one`, lens[] holds append offsets and the length is offset + 1.
__device__ void tile_prefix(const int64_t* __restrict__ lens, int B, int64_t cap, int TT, int* prefix,
                            int* lens_s, int* warp_sums, int plus_one = 0) {
    const int tid = threadIdx.x, nthreads = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int per = (B + nthreads - 1) / nthreads;
    const int lo = min(B, tid * per), hi = min(B, lo + per);
    int local = 0;
    for (int i = lo; i < hi; ++i) {
        const int64_t len = lens[i] + plus_one;
        const int usable = (len > 0 && len <= cap) ? (int)len : 0;
        lens_s[i] = usable;
        local += (usable + TT - 1) / TT;
    }
    int incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        const int nw = nthreads >> 5;
        int w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, w, off);
            if (lane >= off) w += v;
        }
        if (lane < nw) warp_sums[lane] = w;  // inclusive
    }
    __syncthreads();
    int run = incl - local + (warp > 0 ? warp_sums[warp - 1] : 0);
    for (int i = lo; i < hi; ++i) {
        prefix[i] = run;
        run += (lens_s[i] + TT - 1) / TT;
    }
    if (tid == nthreads - 1) prefix[B] = run;
    __syncthreads();
}

// Largest b in [0, B) with prefix[b] <= t (the request owning tile t).
__device__ __forceinline__ int request_of_tile(const int* prefix, int B, int t) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
    }
    return lo;
}

// One warp merges the partial records of request b for query heads qh0 and
// (when two is set) qh0 + 1: records b + c for the CTAs c in [c0, c1] that own
// tiles.  Online over chunks of four records: every load of a chunk (the
// log-sum-exps and the partial rows of both heads) is issued before any of it
// is combined, so the merge of a request split over k CTAs costs ceil(k / 4)
// rounds of L2 loads for two heads.  Records of empty segments have lse = -inf
// and weigh nothing.
template <typename T, int D>
__device__ void merge_heads(const DecodeParams& p, int b, int qh0, bool two, int c0, int c1, int G, int total,
                            int lane) {
    constexpr int kBatch = (sizeof(T) == 2 && D <= 128) ? 6 : 4;  // one load round for the typical record count
    constexpr int kDims = (D + 31) / 32;
    const int nh = two ? 2 : 1;
    const int n = c1 - c0 + 1;
    const int64_t first = (int64_t)b + c0;
    float m_run[2] = {-INFINITY, -INFINITY}, wsum[2] = {0.f, 0.f};
    float acc[2][kDims];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < kDims; ++i) acc[h][i] = 0.f;
    for (int k0 = 0; k0 < n; k0 += kBatch) {
        float lse[2][kBatch];
        float vals[2][kBatch][kDims];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int k = k0 + u;
            const bool use = k < n && cta_owns_tiles(c0 + k, G, total);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const bool on = use && h < nh;
                const int64_t rec = (first + k) * p.q_heads + qh0 + h;
                lse[h][u] = on ? __ldcg(p.lse + rec) : -INFINITY;
                const float* part = p.partial + rec * D;
#pragma unroll
                for (int i = 0; i < kDims; ++i) {
                    const int d = lane + 32 * i;
                    vals[h][u][i] = (on && d < D) ? __ldcg(part + d) : 0.f;
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float cm = -INFINITY;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) cm = fmaxf(cm, lse[h][u]);
            const float m_new = fmaxf(m_run[h], cm);
            if (m_new == -INFINITY) continue;
            const float keep = (m_run[h] == -INFINITY) ? 0.f : exp2f(m_run[h] - m_new);
            wsum[h] *= keep;
#pragma unroll
            for (int i = 0; i < kDims; ++i) acc[h][i] *= keep;
#pragma unroll
            for (int u = 0; u < kBatch; ++u) {
                const float w = (lse[h][u] == -INFINITY) ? 0.f : exp2f(lse[h][u] - m_new);
                wsum[h] += w;
#pragma unroll
                for (int i = 0; i < kDims; ++i) acc[h][i] = fmaf(w, vals[h][u][i], acc[h][i]);
            }
            m_run[h] = m_new;
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (h >= nh) break;
        T* out = static_cast<T*>(p.out) + ((int64_t)b * p.q_heads + qh0 + h) * D;
#pragma unroll
        for (int i = 0; i < kDims; ++i) {
            const int d = lane + 32 * i;
            if (d < D) out[d] = Elem<T>::from_float(wsum[h] > 0.f ? acc[h][i] / wsum[h] : 0.f);
        }
    }
}

template <typename T, int D>
struct CoreShape {
    static constexpr int E = Elem<T>::kPerVec;           // elements per 16 B
    static constexpr int VR = D / E;                      // vectors per head row
    static constexpr int LPT = (VR % 8 == 0) ? 8 : (VR % 4 == 0) ? 4 : 2;  // lanes per token
    static constexpr int VPL = VR / LPT;                  // vectors per lane
    static constexpr int TPI = 32 / LPT;                  // lane groups (tokens in flight)
    static constexpr int SC = kTokensPerGroup * TPI;      // tokens per sub-chunk
    static_assert(VR % LPT == 0 && VR >= 2, "unsupported head_dim for this dtype");
};

// ------------------------------------------------------- CUDA-core consumer
// Lane group g (LPT lanes) handles tokens g, g+TPI, ... of each sub-chunk with
// its own online softmax; groups merge when the segment ends.
template <typename T, int D>
struct CoreConsumer {
    using S = CoreShape<T, D>;
    static constexpr int kSubTokens = S::SC;
    static constexpr int kKvBytes = (int)sizeof(T);  // bytes per cached element
    static constexpr bool kPairCapable = false;      // rows staged one per stride
    float qf[kCoreHeads][S::VPL][S::E];
    float acc[kCoreHeads][S::VPL][S::E];
    float m[kCoreHeads], l[kCoreHeads];
    int g, lj;

    __device__ void setup(int lane) {
        g = lane / S::LPT;
        lj = lane % S::LPT;
    }

    __device__ void begin(const T* qrows, int item_heads) {
#pragma unroll
        for (int h = 0; h < kCoreHeads; ++h) {
            const uint4* qrow = reinterpret_cast<const uint4*>(qrows + min(h, item_heads - 1) * D);
#pragma unroll
            for (int v = 0; v < S::VPL; ++v) {
                Elem<T>::load(qrow[lj + v * S::LPT], qf[h][v]);
#pragma unroll
                for (int e = 0; e < S::E; ++e) acc[h][v][e] = 0.f;
            }
            m[h] = -INFINITY;
            l[h] = 0.f;
        }
    }

    __device__ void tile(const unsigned char* ks, const unsigned char* vs, int stride, int TT, int n,
                         uint64_t mask, float scale_log2, bool = false) {
        for (int sub = 0; sub < TT; sub += S::SC) {
            float s[kTokensPerGroup][kCoreHeads];
            bool ok[kTokensPerGroup];
#pragma unroll
            for (int i = 0; i < kTokensPerGroup; ++i) {
                const int j = sub + i * S::TPI + g;
                ok[i] = j < n && ((mask >> j) & 1ull);
                float dot[kCoreHeads];
#pragma unroll
                for (int h = 0; h < kCoreHeads; ++h) dot[h] = 0.f;
                if (ok[i]) {
                    const uint4* row = reinterpret_cast<const uint4*>(ks + j * stride);
#pragma unroll
                    for (int v = 0; v < S::VPL; ++v) {
                        float f[S::E];
                        Elem<T>::load(row[lj + v * S::LPT], f);
#pragma unroll
                        for (int h = 0; h < kCoreHeads; ++h)
#pragma unroll
                            for (int e = 0; e < S::E; ++e) dot[h] = fmaf(qf[h][v][e], f[e], dot[h]);
                    }
                }
#pragma unroll
                for (int off = 1; off < S::LPT; off <<= 1)
#pragma unroll
                    for (int h = 0; h < kCoreHeads; ++h) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], off);
#pragma unroll
                for (int h = 0; h < kCoreHeads; ++h) s[i][h] = ok[i] ? dot[h] * scale_log2 : -INFINITY;
            }
            float pr[kTokensPerGroup][kCoreHeads];
#pragma unroll
            for (int h = 0; h < kCoreHeads; ++h) {
                float mt = s[0][h];
#pragma unroll
                for (int i = 1; i < kTokensPerGroup; ++i) mt = fmaxf(mt, s[i][h]);
                const float mn = fmaxf(m[h], mt);
                float alpha = 1.f, sum = 0.f;
                if (mn != -INFINITY) {
                    alpha = exp2f(m[h] - mn);
#pragma unroll
                    for (int i = 0; i < kTokensPerGroup; ++i) {
                        pr[i][h] = exp2f(s[i][h] - mn);
                        sum += pr[i][h];
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < kTokensPerGroup; ++i) pr[i][h] = 0.f;
                }
                l[h] = l[h] * alpha + sum;
                m[h] = mn;
#pragma unroll
                for (int v = 0; v < S::VPL; ++v)
#pragma unroll
                    for (int e = 0; e < S::E; ++e) acc[h][v][e] *= alpha;
            }
#pragma unroll
            for (int i = 0; i < kTokensPerGroup; ++i) {
                if (!ok[i]) continue;
                const int j = sub + i * S::TPI + g;
                const uint4* row = reinterpret_cast<const uint4*>(vs + j * stride);
#pragma unroll
                for (int v = 0; v < S::VPL; ++v) {
                    float f[S::E];
                    Elem<T>::load(row[lj + v * S::LPT], f);
#pragma unroll
                    for (int h = 0; h < kCoreHeads; ++h)
#pragma unroll
                        for (int e = 0; e < S::E; ++e) acc[h][v][e] = fmaf(pr[i][h], f[e], acc[h][v][e]);
                }
            }
        }
    }

    // Merge lane groups, normalise, write the final row or the partial record.
    __device__ void finish(const DecodeParams& p, int b, int qh0, int item_heads, bool final_row, int64_t record) {
#pragma unroll
        for (int h = 0; h < kCoreHeads; ++h) {
            float mx = m[h];
#pragma unroll
            for (int off = S::LPT; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float f = (m[h] == -INFINITY) ? 0.f : exp2f(m[h] - mx);
            float L = l[h] * f;
#pragma unroll
            for (int off = S::LPT; off < 32; off <<= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
#pragma unroll
            for (int v = 0; v < S::VPL; ++v)
#pragma unroll
                for (int e = 0; e < S::E; ++e) {
                    float a = acc[h][v][e] * f;
#pragma unroll
                    for (int off = S::LPT; off < 32; off <<= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
                    acc[h][v][e] = (L > 0.f) ? a / L : 0.f;
                }
            if (g != 0 || h >= item_heads) continue;
            const int qh = qh0 + h;
            if (final_row) {
                uint4* orow = reinterpret_cast<uint4*>(static_cast<T*>(p.out) + ((int64_t)b * p.q_heads + qh) * D);
#pragma unroll
                for (int v = 0; v < S::VPL; ++v) orow[lj + v * S::LPT] = Elem<T>::store(acc[h][v]);
            } else {
                float4* prow = reinterpret_cast<float4*>(p.partial + (record * p.q_heads + qh) * D);
#pragma unroll
                for (int v = 0; v < S::VPL; ++v)
#pragma unroll
                    for (int e = 0; e < S::E; e += 4)
                        prow[((lj + v * S::LPT) * S::E + e) / 4] =
                            make_float4(acc[h][v][e], acc[h][v][e + 1], acc[h][v][e + 2], acc[h][v][e + 3]);
                if (lj == 0) p.lse[record * p.q_heads + qh] = (L > 0.f) ? mx + log2f(L) : -INFINITY;
            }
        }
    }
};

}  // namespace minikv

#include "decode_mma.cu"

namespace minikv {

// -------------------------------------------------------------- the kernel
template <typename T, int D, typename Consumer>
__global__ void __launch_bounds__(kDecodeThreads, 1) paged_decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int warp_sums[kDecodeThreads / 32];
    __shared__ int last_ticket;
    __shared__ __align__(8) uint64_t seg_bar;  // consumers -> ticket warp: a mid-range partial is stored

    const int TT = p.tile_tokens, NS = p.stages, stride = p.row_stride;
    const int B = p.batch;
    const bool kPair = Consumer::kPairCapable && p.pair_rows;
    const int tile_bytes = kPair ? (TT / 2) * stride : TT * stride;  // K (or V) bytes of one staged tile
    const int stage_bytes = 2 * tile_bytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * stage_bytes);
    uint64_t* empty = full + NS;
    uint64_t* masks = empty + NS;
    int* window = reinterpret_cast<int*>(masks + NS);    // [kWindowTiles][TT] physical rows (-1: masked)
    int* prefix = window + kWindowTiles * TT;             // [B + 1]
    int* lens_s = prefix + B + 1;                         // [B]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t cap = (int64_t)p.table_width * p.block_size;

    // Chained launch: with early_prologue the lengths, the tile split and the
    // page-table reads below overlap the previous kernel (the KV append of the
    // same step), and the wait comes just before the first KV copy / q read.
    if (!p.early_prologue) griddep_wait();
    // The next chained kernel (a projection) may start on SMs that CTAs of this
    // one leave and stream its weights; it waits for this grid before reading
    // what the grid writes.
    griddep_launch_dependents();
    tile_prefix(p.lens, B, cap, TT, prefix, lens_s, warp_sums, p.append);
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init(&seg_bar, kConsumerWarps);
        mbar_init_fence();
    }
    __syncthreads();

    const int total = prefix[B];
    const int G = gridDim.x, c = blockIdx.x;
    if (p.early_prologue && warp < kConsumerWarps) griddep_wait();
    // Requests with no usable tokens get zero rows (reference: count 0 -> 0).
    if (blockIdx.y == 0 && warp < kConsumerWarps) {
        for (int b = c; b < B; b += G) {
            if (lens_s[b] != 0) continue;
            T* row = static_cast<T*>(p.out) + (int64_t)b * p.q_heads * D;
            for (int i = tid; i < p.q_heads * D; i += kConsumerWarps * 32) row[i] = Elem<T>::from_float(0.f);
        }
    }
    const int tile_lo = (int)((int64_t)c * total / G), tile_hi = (int)((int64_t)(c + 1) * total / G);
    if (tile_lo >= tile_hi) return;

    // Head group of this CTA, and the kv head / query-head chunk of consumer warp w.
    const int cph = p.chunks_per_head;
    const int h0 = cph >= kConsumerWarps ? blockIdx.y / p.chunk_groups : blockIdx.y * p.heads_per_cta;
    const int nh = cph >= kConsumerWarps ? 1 : min(p.heads_per_cta, p.kv_heads - h0);
    auto warp_heads = [&](int w, int& kvh_w, int& chunk_w) -> bool {
        if (cph >= kConsumerWarps) {
            kvh_w = h0;
            chunk_w = (blockIdx.y % p.chunk_groups) * kConsumerWarps + w;
            return chunk_w < cph;
        }
        kvh_w = h0 + w / cph;
        chunk_w = w % cph;
        return w < nh * cph;
    };
    int kvh, chunk;
    const bool active = warp_heads(warp, kvh, chunk);
    constexpr int esize = Consumer::kKvBytes;  // bytes per cached element
    const int copy_row = nh * D * esize;              // bytes per token and K|V
    const int cache_row = p.kv_heads * D * esize;     // global row stride

    if (warp == kTicketWarp) {
        // ------------------------------------------------------------ ticket warp
        // Walks the CTA's segments like the consumers; for each one that ends inside
        // the range and is not a whole request, it waits until the consumers have
        // stored the partial (seg_bar, a CTA-scope release/acquire) and takes the
        // request's ticket (acquire-release at GPU scope, cumulative over those
        // stores).  The holder of the last ticket merges every query head of the
        // CTA's head group, while the consumers already stream the next request.
        griddep_wait();  // tickets and outputs may still be in use by the previous kernel
        int k = 0;
        int b = request_of_tile(prefix, B, tile_lo);
        for (int t = tile_lo; t < tile_hi;) {
            while (b + 1 < B && prefix[b + 1] <= t) ++b;
            const int seg_hi = min(tile_hi, prefix[b + 1]);
            const int c0 = cta_of_tile(prefix[b], G, total), c1 = cta_of_tile(prefix[b + 1] - 1, G, total);
            if (c0 != c1 && seg_hi < tile_hi) {
                mbar_wait(&seg_bar, k & 1);  // on a timeout the ticket is still taken: the counter stays consistent
                ++k;
                int owners = 0;
                for (int cc = c0; cc <= c1; ++cc) owners += cta_owns_tiles(cc, G, total) ? 1 : 0;
                unsigned int ticket = 0;
                if (lane == 0)
                    asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                                 : "=r"(ticket)
                                 : "l"(p.tickets + (int64_t)b * gridDim.y + blockIdx.y),
                                   "r"((unsigned int)(owners - 1))
                                 : "memory");
                ticket = __shfl_sync(0xffffffffu, ticket, 0);
                __syncwarp();  // the other lanes' partial loads come after lane 0's acquire
                if (ticket == (unsigned int)(owners - 1)) {
                    for (int w = 0; w < kConsumerWarps; ++w) {
                        int kvh_w, chunk_w;
                        if (!warp_heads(w, kvh_w, chunk_w)) continue;
                        const int ih = min(p.heads_per_item, p.group - chunk_w * p.heads_per_item);
                        const int qh_w = kvh_w * p.group + chunk_w * p.heads_per_item;
                        for (int h = 0; h < ih; h += 2)
                            merge_heads<T, D>(p, b, qh_w + h, h + 1 < ih, c0, c1, G, total, lane);
                    }
                }
            }
            t = seg_hi;
        }
        return;
    }

    if (warp == kProducerWarp) {
        // ------------------------------------------------------------ producer
        const uint64_t policy = policy_evict_first();
        const uint64_t space_limit = space_wait_limit();
        const unsigned char* kbase = static_cast<const unsigned char*>(p.kc) + (size_t)h0 * D * esize;
        const unsigned char* vbase = static_cast<const unsigned char*>(p.vc) + (size_t)h0 * D * esize;
        const uint64_t tile_bits = (TT == 64) ? ~0ull : ((1ull << TT) - 1);
        // fused append: the new rows of this CTA's heads (row stride: every kv head of a request)
        const int new_row = p.kv_heads * D * esize;
        const unsigned char* knew = static_cast<const unsigned char*>(p.new_k) + (size_t)h0 * D * esize;
        const unsigned char* vnew = static_cast<const unsigned char*>(p.new_v) + (size_t)h0 * D * esize;
        int gt = 0;            // tiles issued
        bool stopped = false;  // a space wait gave up: issue nothing more
        bool waited = !p.early_prologue;  // griddepcontrol.wait done (or not needed)
        for (int w0 = tile_lo; w0 < tile_hi && !stopped; w0 += kWindowTiles) {
            // Rows of tiles w0 .. w0+31: lane i resolves tile w0+i, one table
            // load per page, all lanes' loads in flight together.
            const int t = w0 + lane;
            int append_dst = -1, append_b = 0;  // fused append: pool row this lane's tile writes, its request
            if (t < tile_hi) {
                const int b = request_of_tile(prefix, B, t);
                const int k = t - prefix[b];
                const int64_t t0 = (int64_t)k * TT;
                const int n = (int)min((int64_t)TT, (int64_t)lens_s[b] - t0);
                const int64_t* table = p.tables + (p.table_rows ? p.table_rows[b] : (int64_t)b) * p.table_width;
                int* rows = window + lane * TT;
                int j = 0;
                while (j < n) {
                    const int64_t pos = t0 + j;
                    const int64_t page = table[pos / p.block_size];
                    const int in_page = (int)(pos % p.block_size);
                    const int run = min(n - j, p.block_size - in_page);
                    const bool ok = page >= 0 && page < p.num_blocks;
                    const int base = ok ? (int)(page * p.block_size) + in_page : -1;
                    for (int r = 0; r < run; ++r) rows[j + r] = ok ? base + r : -1;
                    j += run;
                }
                // Fused append: the last token of the request's last tile is the new one.  It is
                // staged from the source row (entry -2 - b) and written to its pool row below.
                if (p.append && t0 + n == lens_s[b] && rows[n - 1] >= 0) {
                    append_dst = rows[n - 1];
                    append_b = b;
                    // 16-bit pools stage the new row from its source; an fp8 pool stages it from the
                    // pool once it has been quantised there (below, before its tile is issued)
                    if constexpr (esize != 1) rows[n - 1] = -2 - b;
                }
                for (; j < TT; ++j) rows[j] = -1;
            }
            __syncwarp();
            // Chained launch: the copies wait for the previous kernel (the KV rows may come from
            // it).  With the fused append they need not: the pool rows it reads predate the
            // previous kernel and only the new rows (read from key/value) may come from it, so
            // the copies start at once and the wait comes before the first new row, before the
            // producer would block on a full ring, and before the new rows are written back.
            if (!waited && !(p.append && p.early_prologue)) {
                griddep_wait();
                waited = true;
            }
            const int count = min(kWindowTiles, tile_hi - w0);
            for (int i = 0; i < count; ++i, ++gt) {
                const int slot = gt % NS;
                if (gt >= NS && !waited) {  // a full ring: the consumers start only after the previous kernel
                    griddep_wait();
                    waited = true;
                }
                if (gt >= NS && !__all_sync(0xffffffffu, mbar_wait_space(&empty[slot], ((gt / NS) - 1) & 1, space_limit))) {
                    stopped = true;  // the consumers may still read this slot
                    break;
                }
                int row[2];
                bool ok[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int j = lane + 32 * h;
                    row[h] = j < TT ? window[i * TT + j] : -1;
                    ok[h] = row[h] != -1;  // a pool row, or (append) -2 - b: request b's new row
                }
                if (!waited && __any_sync(0xffffffffu, row[0] < -1 || row[1] < -1)) {  // a new row: from the previous kernel
                    griddep_wait();
                    waited = true;
                }
                if constexpr (esize == 1) {
                    // fused append into an fp8 pool: quantise the tile's new row into its pool slot,
                    // then order those generic stores before the bulk copies that read the slot
                    const int new_dst = __shfl_sync(0xffffffffu, append_dst, i);
                    if (p.append && new_dst >= 0) {
                        const int64_t src = __shfl_sync(0xffffffffu, append_b, i);
                        if (!waited) {
                            griddep_wait();
                            waited = true;
                        }
                        unsigned char* kpool = const_cast<unsigned char*>(kbase) + (int64_t)new_dst * cache_row;
                        unsigned char* vpool = const_cast<unsigned char*>(vbase) + (int64_t)new_dst * cache_row;
                        const T* ks = static_cast<const T*>(p.new_k) + (src * p.kv_heads + h0) * D;
                        const T* vs = static_cast<const T*>(p.new_v) + (src * p.kv_heads + h0) * D;
                        quantize_row_warp<T, Consumer::kE5M2>(kpool, ks, copy_row, p.k_inv, lane);
                        quantize_row_warp<T, Consumer::kE5M2>(vpool, vs, copy_row, p.v_inv, lane);
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                        __syncwarp();
                    }
                }
                const uint64_t mask = (uint64_t)__ballot_sync(0xffffffffu, ok[0]) |
                                      ((uint64_t)__ballot_sync(0xffffffffu, ok[1]) << 32);
                unsigned char* kdst = smem + slot * stage_bytes;
                unsigned char* vdst = kdst + tile_bytes;
                // Masked V rows must hold finite values (the tensor-core PV
                // multiplies them by P = 0): zero them with generic stores,
                // ordered before the consumers' reads by the arrive below.
                uint64_t holes = ~mask & tile_bits;
                while (holes) {
                    const int j = __ffsll((long long)holes) - 1;
                    holes &= holes - 1;
                    uint4* vrow = reinterpret_cast<uint4*>(vdst + stage_row_offset(kPair, j, stride, copy_row));
                    for (int v = lane; v < copy_row / 16; v += 32) vrow[v] = make_uint4(0, 0, 0, 0);
                }
                __syncwarp();
                if (lane == 0) {
                    masks[slot] = mask;
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)(__popcll(mask) * copy_row * 2));
                }
                __syncwarp();
                if (p.coalesce) {
                    // A run = consecutive tokens whose physical rows are consecutive: one
                    // copy of len rows (stride == copy_row == cache_row here).
                    const int prev0 = __shfl_up_sync(0xffffffffu, row[0], 1);
                    const int last0 = __shfl_sync(0xffffffffu, row[0], 31);
                    const int prev1 = __shfl_up_sync(0xffffffffu, row[1], 1);
                    const bool head0 = ok[0] && (lane == 0 || prev0 < 0 || prev0 != row[0] - 1);
                    const bool head1 = ok[1] && (lane == 0 ? (last0 < 0 || last0 != row[1] - 1)
                                                           : (prev1 < 0 || prev1 != row[1] - 1));
                    const uint64_t heads = (uint64_t)__ballot_sync(0xffffffffu, head0) |
                                           ((uint64_t)__ballot_sync(0xffffffffu, head1) << 32);
                    const uint64_t stops = heads | ~mask;  // bits >= TT are never in mask
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (!(h ? head1 : head0)) continue;
                        const int j = lane + 32 * h;
                        const uint64_t rest = j < 63 ? (stops >> (j + 1)) : 0ull;
                        const int len = rest ? __ffsll((long long)rest) : 64 - j;
                        const int64_t r = row[h];
                        bulk_load(kdst + j * stride, kbase + r * cache_row, (uint32_t)(len * copy_row), &full[slot],
                                  policy);
                        bulk_load(vdst + j * stride, vbase + r * cache_row, (uint32_t)(len * copy_row), &full[slot],
                                  policy);
                    }
                } else {
                    // Paired staging: two consecutive tokens whose pool rows are consecutive (the
                    // same page) go in one copy of two rows, issued by the even token's lane.
                    int partner[2];
#pragma unroll
                    for (int h = 0; h < 2; ++h) partner[h] = __shfl_xor_sync(0xffffffffu, row[h], 1);
                    const bool even = (lane & 1) == 0;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (!ok[h]) continue;
                        const bool paired = kPair && (even ? (row[h] >= 0 && partner[h] == row[h] + 1)
                                                           : (partner[h] >= 0 && row[h] == partner[h] + 1));
                        if (paired && !even) continue;  // copied with the even token
                        const int j = lane + 32 * h;
                        const int64_t r = row[h];
                        const unsigned char* ksrc = r >= 0 ? kbase + r * cache_row : knew + (-2 - r) * new_row;
                        const unsigned char* vsrc = r >= 0 ? vbase + r * cache_row : vnew + (-2 - r) * new_row;
                        const int off = stage_row_offset(kPair, j, stride, copy_row);
                        const uint32_t bytes = (uint32_t)(paired ? 2 * copy_row : copy_row);
                        bulk_load(kdst + off, ksrc, bytes, &full[slot], policy);
                        bulk_load(vdst + off, vsrc, bytes, &full[slot], policy);
                    }
                }
            }
            __syncwarp();
            if (esize != 1 && p.append) {  // (an fp8 pool's new rows were written before their tiles)
                if (!waited) {
                    griddep_wait();
                    waited = true;
                }
                // write this window's appended rows (this CTA's heads) into the pool: every
                // lane copies 16 bytes at a time of one row after the other; bit-exact copies
                unsigned pending = __ballot_sync(0xffffffffu, append_dst >= 0);
                unsigned char* kpool = const_cast<unsigned char*>(kbase);
                unsigned char* vpool = const_cast<unsigned char*>(vbase);
                while (pending) {
                    const int from = __ffs(pending) - 1;
                    pending &= pending - 1;
                    const int64_t dst = __shfl_sync(0xffffffffu, append_dst, from);
                    const int64_t src = __shfl_sync(0xffffffffu, append_b, from);
                    const uint4* ks = reinterpret_cast<const uint4*>(knew + src * new_row);
                    const uint4* vs = reinterpret_cast<const uint4*>(vnew + src * new_row);
                    uint4* kd = reinterpret_cast<uint4*>(kpool + dst * cache_row);
                    uint4* vd = reinterpret_cast<uint4*>(vpool + dst * cache_row);
                    for (int v = lane; v < copy_row / 16; v += 32) {
                        kd[v] = ld_global_nc(ks + v);
                        vd[v] = ld_global_nc(vs + v);
                    }
                }
            }
        }
        // Drain: the last phase issued into each slot has landed before this warp
        // exits, so no bulk copy is in flight when the CTA releases its shared memory
        // (on the normal path these phases are complete or about to be).
        if (lane == 0)
            for (int s2 = 0; s2 < NS && s2 < gt; ++s2) mbar_drain(&full[s2], ((s2 + NS * ((gt - 1 - s2) / NS)) / NS) & 1);
        __syncwarp();
        return;
    }

    // ---------------------------------------------------------------- consumers
    Consumer cons;
    cons.setup(lane);
    const int item_heads = min(p.heads_per_item, p.group - chunk * p.heads_per_item);
    const int local_head = kvh - h0;
    const int qh0 = kvh * p.group + chunk * p.heads_per_item;
    int gt = 0;
    int b = request_of_tile(prefix, B, tile_lo);
    for (int t = tile_lo; t < tile_hi;) {
        while (b + 1 < B && prefix[b + 1] <= t) ++b;
        const int seg_hi = min(tile_hi, prefix[b + 1]);
        const int len = lens_s[b];
        if (active) cons.begin(static_cast<const T*>(p.q) + ((int64_t)b * p.q_heads + qh0) * D, item_heads);
        for (int k = t - prefix[b]; k < seg_hi - prefix[b]; ++k, ++gt) {
            const int slot = gt % NS;
            // a stage whose wait gave up is skipped (its copies may still be landing); the
            // arrival below still happens, so the ticket protocol and the ring stay consistent
            const bool landed = __all_sync(0xffffffffu, mbar_wait(&full[slot], (gt / NS) & 1));
            if (active && landed) {
                const unsigned char* ks = smem + slot * stage_bytes + local_head * D * esize;
                cons.tile(ks, ks + tile_bytes, stride, TT, min(TT, len - k * TT), masks[slot], p.scale_log2, kPair);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        const int c0 = cta_of_tile(prefix[b], G, total), c1 = cta_of_tile(prefix[b + 1] - 1, G, total);
        const bool final_row = c0 == c1;
        if (active) cons.finish(p, b, qh0, item_heads, final_row, (int64_t)b + c);
        if (!final_row && seg_hi < tile_hi) {
            // a request boundary inside the range: the ticket warp takes the ticket
            __syncwarp();  // the warp's partial stores before lane 0's release
            if (lane == 0) mbar_arrive(&seg_bar);
        } else if (!final_row) {
            // Ticket: the CTA that completes request b last merges its records.
            // The consumer barrier orders every thread's partial stores before
            // thread 0's ticket, an acquire-release atomic at GPU scope: it
            // publishes this CTA's records (release, cumulative over the
            // barrier) and, for the last ticket, makes the other CTAs' records
            // visible to this CTA once the second barrier has passed (acquire).
            int owners = 0;
            for (int cc = c0; cc <= c1; ++cc) owners += cta_owns_tiles(cc, G, total) ? 1 : 0;
            consumers_sync();
            if (tid == 0) {
                unsigned int ticket;
                asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;"
                             : "=r"(ticket)
                             : "l"(p.tickets + (int64_t)b * gridDim.y + blockIdx.y), "r"((unsigned int)(owners - 1))
                             : "memory");
                last_ticket = (ticket == (unsigned int)(owners - 1)) ? 1 : 0;
            }
            consumers_sync();
            if (last_ticket) {
                if (active)
                    for (int h = 0; h < item_heads; h += 2)
                        merge_heads<T, D>(p, b, qh0 + h, h + 1 < item_heads, c0, c1, G, total, lane);
            }
            consumers_sync();  // last_ticket is reused by the next segment
        }
        t = seg_hi;
    }
}

// ------------------------------------------------------------------ host side
struct DecodePlan {
    bool mma, coalesce, pair_rows;
    int tile_tokens, stages, row_stride, heads_per_item, heads_per_cta, chunks_per_head, chunk_groups,
        head_groups;
    int grid, smem_bytes;
    int64_t records, ws_tickets, ws_lse, ws_partial, ws_bytes;
};

static int esize_of(int dtype) { return dtype == 0 ? 4 : 2; }

static int lanes_per_token(int D, int esize) {
    const int vr = D * esize / 16;
    return (vr % 8 == 0) ? 8 : (vr % 4 == 0) ? 4 : 2;
}

static int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// Everything here depends on shapes and the device only (graph-static).
static bool make_decode_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size,
                             int64_t table_width, int dtype, int sm_count, DecodePlan* plan,
                             bool kv_fp8 = false) {
    // kv_fp8: one-byte (e4m3) pool read by the fp8 tensor-core consumer (decode_fp8.cu)
    const int es = kv_fp8 ? 1 : esize_of(dtype);
    const bool mma = kv_fp8 || dtype != 0;
    const int sc = mma ? 16 : kTokensPerGroup * (32 / lanes_per_token((int)D, es));
    const int heads_per_item = mma ? kMmaHeads : kCoreHeads;
    const int64_t group = Hq / Hkv;
    const int cph = (int)((group + heads_per_item - 1) / heads_per_item);
    int hpc, ncg, z;
    if (cph >= kConsumerWarps) {
        hpc = 1;
        ncg = (cph + kConsumerWarps - 1) / kConsumerWarps;
        z = (int)Hkv * ncg;
    } else {
        const int by_row = (int)std::max<int64_t>(1, 2048 / (D * es));
        hpc = (int)std::min<int64_t>({Hkv, (int64_t)(kConsumerWarps / cph), (int64_t)by_row});
        ncg = 1;
        z = (int)((Hkv + hpc - 1) / hpc);
    }
    // Padding by 16 bytes makes (stride / 16) odd: ldmatrix rows hit distinct banks.
    // fp8 pool with every kv head in one CTA: token rows are contiguous in the
    // pool, so they are staged unpadded and copied in runs (the fp8 consumer's
    // loads are built for that layout).
    // 16-bit pools on the tensor-core consumer stage rows in pairs (one copy per two tokens of a
    // page, padding after each pair; the consumer reads even and odd tokens as separate 8-row
    // groups, which keeps ldmatrix conflict free).
    const bool coalesce = kv_fp8 && hpc == Hkv;
    const bool pair = mma && !kv_fp8 && hpc == Hkv;  // a pair of rows is contiguous in the pool
    const int row_bytes = hpc * (int)D * es;
    const int stride = pair ? 2 * row_bytes + 16 : row_bytes + (coalesce ? 0 : 16);
    const int token_bytes = pair ? stride / 2 : stride;
    int tt = (32768 / token_bytes) / sc * sc;
    tt = std::max(sc, std::min(64, tt));
    const int stage = 2 * (pair ? (tt / 2) * stride : tt * stride);
    const int fixed = kWindowTiles * tt * 4 + (int)(2 * B + 1) * 4 + 128;
    const int max_smem = 232448 - 1024;  // opt-in limit per block, minus static shared memory
    int stages = std::min(kv_fp8 ? 6 : 4, (196608 + 8192) / stage);
    while (stages > 1 && stages * (stage + 24) + fixed > max_smem) --stages;
    if (stages < 1 || stages * (stage + 24) + fixed > max_smem) return false;
    const int smem = stages * (stage + 24) + fixed;
    const int per_sm = std::max(1, std::min(2, 227 * 1024 / (smem + 1024)));
    const int64_t cap = table_width * block_size;
    const int64_t upper_tiles = B * ((cap + tt - 1) / tt);
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((int64_t)sm_count * per_sm, upper_tiles));
    plan->mma = mma;
    plan->tile_tokens = tt;
    plan->stages = stages;
    plan->row_stride = stride;
    plan->pair_rows = pair;
    plan->coalesce = coalesce;
    plan->heads_per_item = heads_per_item;
    plan->heads_per_cta = hpc;
    plan->chunks_per_head = cph;
    plan->chunk_groups = ncg;
    plan->head_groups = z;
    plan->grid = (int)grid;
    plan->smem_bytes = smem;
    plan->records = B + grid - 1;
    plan->ws_tickets = 0;
    plan->ws_lse = align256(B * z * 4);
    plan->ws_partial = plan->ws_lse + align256(plan->records * Hq * 4);
    plan->ws_bytes = plan->ws_partial + align256(plan->records * Hq * D * 4);
    return true;
}

template <typename T, int D>
static cudaError_t launch_decode_typed(const DecodeParams& p, const DecodePlan& plan, cudaStream_t stream) {
    using Consumer = typename std::conditional<sizeof(T) == 2, MmaConsumer<T, D>, CoreConsumer<T, D>>::type;
    auto kernel = paged_decode_kernel<T, D, Consumer>;
    // the opt-in shared-memory size, raised once per device and size (a host call per launch otherwise)
    static int configured[64] = {0};
    cudaError_t err = ensure_smem_limit(kernel, plan.smem_bytes, configured);
    if (err != cudaSuccess) return err;
    return launch_chained(kernel, dim3(plan.grid, plan.head_groups), dim3(kDecodeThreads), plan.smem_bytes, stream, p);
}

template <typename T>
static cudaError_t launch_decode_dim(int D, const DecodeParams& p, const DecodePlan& plan, cudaStream_t stream) {
    switch (D) {
        case 16: return launch_decode_typed<T, 16>(p, plan, stream);
        case 32: return launch_decode_typed<T, 32>(p, plan, stream);
        case 64: return launch_decode_typed<T, 64>(p, plan, stream);
        case 80: return launch_decode_typed<T, 80>(p, plan, stream);
        case 96: return launch_decode_typed<T, 96>(p, plan, stream);
        case 128: return launch_decode_typed<T, 128>(p, plan, stream);
        case 192: return launch_decode_typed<T, 192>(p, plan, stream);
        case 256: return launch_decode_typed<T, 256>(p, plan, stream);
        default: return cudaErrorInvalidValue;
    }
}

static cudaError_t launch_decode(int dtype, int D, const DecodeParams& p, const DecodePlan& plan,
                                 cudaStream_t stream) {
    if (dtype == 0) return launch_decode_dim<float>(D, p, plan, stream);
    if (dtype == 1) return launch_decode_dim<__half>(D, p, plan, stream);
    return launch_decode_dim<__nv_bfloat16>(D, p, plan, stream);
}

// Fill DecodeParams from a plan; `tickets`, `lse` and `partial` point into the
// scratch memory `ws` laid out by the plan.
static DecodeParams decode_params(const void* query, const void* key_cache, const void* value_cache,
                                  const int64_t* block_tables, const int64_t* context_lens,
                                  const int64_t* table_rows, void* out, unsigned char* ws, int64_t batch,
                                  int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t num_blocks,
                                  int64_t block_size, int64_t table_width, const DecodePlan& plan) {
    DecodeParams p{};
    p.q = query;
    p.kc = key_cache;
    p.vc = value_cache;
    p.tables = block_tables;
    p.lens = context_lens;
    p.table_rows = table_rows;
    p.out = out;
    p.tickets = reinterpret_cast<unsigned int*>(ws + plan.ws_tickets);
    p.lse = reinterpret_cast<float*>(ws + plan.ws_lse);
    p.partial = reinterpret_cast<float*>(ws + plan.ws_partial);
    p.batch = (int)batch;
    p.q_heads = (int)q_heads;
    p.kv_heads = (int)kv_heads;
    p.num_blocks = (int)std::min<int64_t>(num_blocks, 2147483647);
    p.block_size = (int)block_size;
    p.table_width = (int)table_width;
    p.group = (int)(q_heads / kv_heads);
    p.heads_per_item = plan.heads_per_item;
    p.chunks_per_head = plan.chunks_per_head;
    p.heads_per_cta = plan.heads_per_cta;
    p.chunk_groups = plan.chunk_groups;
    p.tile_tokens = plan.tile_tokens;
    p.stages = plan.stages;
    p.row_stride = plan.row_stride;
    p.pair_rows = plan.pair_rows ? 1 : 0;
    p.coalesce = plan.coalesce ? 1 : 0;
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
    return p;
}

static int run_decode(const void* query, const void* key_cache, const void* value_cache,
                      const int64_t* block_tables, const int64_t* context_lens, const int64_t* table_rows,
                      void* out, void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                      int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                      int64_t table_width, int dtype, cudaStream_t stream, bool early_prologue = false,
                      const void* new_k = nullptr, const void* new_v = nullptr) {
    DecodePlan plan;
    if (!make_decode_plan(batch, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sm_count(), &plan))
        return fail(MINIKV_EUNSUPPORTED, "decode shape does not fit shared memory (batch too large?)");
    MINIKV_REQUIRE(workspace != nullptr && workspace_bytes >= plan.ws_bytes && aligned16(workspace),
                   MINIKV_EINVAL, "decode workspace too small or misaligned");
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    // The ticket region (the first bytes of the workspace) must be zero when
    // the kernel starts; every launch leaves it zero again (atomicInc wraps).
    const DecodeParams p = decode_params(query, key_cache, value_cache, block_tables, context_lens, table_rows,
                                         out, ws, batch, q_heads, kv_heads, head_dim, num_blocks, block_size,
                                         table_width, plan);
    DecodeParams q = p;
    q.early_prologue = early_prologue ? 1 : 0;
    if (new_k != nullptr) {  // fused append: context_lens holds the token offsets
        if (plan.coalesce) return fail(MINIKV_EUNSUPPORTED, "fused KV append needs a 16-bit or fp32 pool");
        q.append = 1;
        q.new_k = new_k;
        q.new_v = new_v;
    }
    const cudaError_t err = launch_decode(dtype, (int)head_dim, q, plan, stream);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_decode launch");
    return MINIKV_OK;
}

// Bytes at the start of a decode workspace that must be zero before its first use.
static int64_t decode_ticket_bytes(const DecodePlan& plan) { return plan.ws_lse; }

}  // namespace minikv
