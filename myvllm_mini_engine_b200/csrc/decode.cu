// Split-KV (flash-decoding) paged decode attention for sm_100a.
//
// Work decomposition ("balanced split-KV").  The tokens of every request are
// cut into tiles of TT tokens; the tiles of the whole batch form one list of
// `total` tiles and CTA c of a persistent grid of G CTAs (one per SM) takes
// tiles [c*total/G, (c+1)*total/G).  A CTA therefore streams an equal share
// of the batch's KV bytes whatever the (ragged) lengths are; its range covers
// one or more request *segments*.  A segment that is a whole request writes
// the final output; otherwise it writes an fp32 partial (output normalised by
// its own softmax sum) and its log2-sum-exp, and a second kernel merges the
// partials of each request (exactly the reference's merge,
// mini_engine/kernels/csrc/paged_attention.cu:195-215).  The grid, the
// workspace and the record layout depend only on (batch, table width, block
// size, heads, head dim, dtype) and the SM count, never on context_lens, so a
// captured CUDA graph stays valid when lengths change (the reference derives
// its partition count from the table width for the same reason,
// paged_attention.cu:271).
//
// CTA layout: 8 consumer warps + 1 producer warp.  The producer stages each
// tile's K and V rows -- all kv heads of the CTA's head group, i.e. whole
// contiguous page rows -- into shared memory with 1-D bulk copies (TMA engine)
// on a ring of `stages` buffers guarded by full/empty mbarriers.  Each
// consumer warp owns one kv head and two of its query heads (GQA: every KV
// byte is read from HBM once per step, whatever the group size), keeps a
// per-lane-group online softmax in registers and merges the lane groups when
// the segment ends.
//
// Trusted-mode guards of the reference kernel are kept: a page id outside
// [0, num_blocks) masks its tokens (score -inf, paged_attention.cu:72-82); a
// length outside [1, table_width*block_size] yields an all-zero row (:62-64);
// a row with no unmasked token yields zeros (:99, :120).
#include "common.cuh"

namespace minikv {

constexpr int kConsumerWarps = 8;
constexpr int kDecodeThreads = (kConsumerWarps + 1) * 32;
constexpr int kItemHeads = 2;      // query heads per consumer warp
constexpr int kTokensPerGroup = 4; // tokens per lane group per sub-chunk

struct DecodeParams {
    const void* q;
    const void* kc;
    const void* vc;
    const int64_t* tables;
    const int64_t* lens;
    const int64_t* table_rows;  // table row of request b (nullptr: row b)
    void* out;
    float* partial;   // [records, q_heads, D]
    float* lse;       // [records, q_heads]   (log2 domain)
    int* prefix_out;  // [batch + 1] tile prefix, written by CTA (0, 0)
    int batch, q_heads, kv_heads, num_blocks, block_size, table_width;
    int group;            // q_heads / kv_heads
    int chunks_per_head;  // ceil(group / kItemHeads)
    int heads_per_cta;    // kv heads per CTA head group (1 when chunks_per_head >= 8)
    int chunk_groups;     // head groups per kv head (> 1 only when chunks_per_head > 8)
    int tile_tokens;      // TT, multiple of the sub-chunk size, <= 64
    int stages;
    int row_bytes;        // shared-memory row stride = heads_per_cta * D * elem
    float scale_log2;     // log2(e) / sqrt(D)
};

template <typename T, int D>
struct DecodeShape {
    static constexpr int E = Elem<T>::kPerVec;           // elements per 16 B
    static constexpr int VR = D / E;                      // vectors per head row
    static constexpr int LPT = (VR % 8 == 0) ? 8 : (VR % 4 == 0) ? 4 : 2;  // lanes per token
    static constexpr int VPL = VR / LPT;                  // vectors per lane
    static constexpr int TPI = 32 / LPT;                  // lane groups (tokens in flight)
    static constexpr int SC = kTokensPerGroup * TPI;      // tokens per sub-chunk
    static_assert(VR % LPT == 0 && VR >= 2, "unsupported head_dim for this dtype");
};

// CTA c of G owns tiles [c*total/G, (c+1)*total/G); cta_of(t) inverts it.
__device__ __forceinline__ int cta_of_tile(int t, int G, int total) {
    return (int)((((int64_t)t + 1) * G + total - 1) / total) - 1;
}

// Exclusive prefix of per-request tile counts into prefix[0..B] (shared).
__device__ void tile_prefix(const int64_t* __restrict__ lens, int B, int64_t cap, int TT, int* prefix,
                            int* warp_sums) {
    const int tid = threadIdx.x, nthreads = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int per = (B + nthreads - 1) / nthreads;
    const int lo = min(B, tid * per), hi = min(B, lo + per);
    int local = 0;
    for (int i = lo; i < hi; ++i) {
        const int64_t len = lens[i];
        local += (len > 0 && len <= cap) ? (int)((len + TT - 1) / TT) : 0;
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
        const int64_t len = lens[i];
        prefix[i] = run;
        run += (len > 0 && len <= cap) ? (int)((len + TT - 1) / TT) : 0;
    }
    if (tid == nthreads - 1) prefix[B] = run;
    __syncthreads();
}

template <typename T, int D>
__global__ void __launch_bounds__(kDecodeThreads, 1) paged_decode_split_kernel(const DecodeParams p) {
    using S = DecodeShape<T, D>;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ int warp_sums[kDecodeThreads / 32];

    const int TT = p.tile_tokens, NS = p.stages, row_bytes = p.row_bytes;
    const int stage_bytes = 2 * TT * row_bytes;
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

    // Head group of this CTA and the query heads of this consumer warp.
    const int cph = p.chunks_per_head;
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
    constexpr int esize = (int)sizeof(T);
    const int copy_row = nh * D * esize;                    // bytes per token and K|V
    const int cache_row = p.kv_heads * D * esize;           // global row stride
    const bool whole_rows = (nh == p.kv_heads);             // CTA rows are contiguous in HBM
    int b = 0;
    {   // request containing tile_lo: largest b with prefix[b] <= tile_lo
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
                if (lane == 0) {
                    masks[slot] = mask;
                    mbar_arrive_expect_tx(&full[slot], (uint32_t)(__popcll(mask) * copy_row * 2));
                }
                __syncwarp();
                unsigned char* kdst = smem + slot * stage_bytes;
                unsigned char* vdst = kdst + TT * row_bytes;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int j = lane + 32 * h;
                    if (!ok[h]) continue;
                    if (whole_rows) {
                        // one copy per run of valid tokens inside one page
                        const bool prev_ok = j > 0 && ((mask >> (j - 1)) & 1ull);
                        const bool page_start = ((t0 + j) % p.block_size) == 0;
                        if (prev_ok && !page_start) continue;
                        const int to_page_end = (int)(p.block_size - (t0 + j) % p.block_size);
                        int end = min(n, j + to_page_end);
                        const uint64_t above = (j >= 63) ? 0ull : (~0ull << (j + 1));
                        const uint64_t gaps = ~mask & above;
                        if (gaps) end = min(end, __ffsll((long long)gaps) - 1);
                        const uint32_t bytes = (uint32_t)((end - j) * copy_row);
                        bulk_load(kdst + j * row_bytes, kbase + rows[h] * cache_row, bytes, &full[slot], policy);
                        bulk_load(vdst + j * row_bytes, vbase + rows[h] * cache_row, bytes, &full[slot], policy);
                    } else {
                        bulk_load(kdst + j * row_bytes, kbase + rows[h] * cache_row, copy_row, &full[slot], policy);
                        bulk_load(vdst + j * row_bytes, vbase + rows[h] * cache_row, copy_row, &full[slot], policy);
                    }
                }
            }
            t = seg_hi;
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int g = lane / S::LPT, lj = lane % S::LPT;
    const int item_heads = min(kItemHeads, p.group - chunk * kItemHeads);
    const int local_head = kvh - h0;
    float qf[kItemHeads][S::VPL][S::E];
    float acc[kItemHeads][S::VPL][S::E];
    float m[kItemHeads], l[kItemHeads];
    int gt = 0;
    for (int t = tile_lo; t < tile_hi;) {
        while (b + 1 < B && prefix[b + 1] <= t) ++b;
        const int seg_hi = min(tile_hi, prefix[b + 1]);
        const int64_t len = p.lens[b];
        if (active) {
#pragma unroll
            for (int h = 0; h < kItemHeads; ++h) {
                const int qh = kvh * p.group + chunk * kItemHeads + min(h, item_heads - 1);
                const uint4* qrow = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) +
                                                                   ((int64_t)b * p.q_heads + qh) * D);
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
        for (int k = t - prefix[b]; k < seg_hi - prefix[b]; ++k, ++gt) {
            const int slot = gt % NS;
            mbar_wait(&full[slot], (gt / NS) & 1);
            if (active) {
                const uint64_t mask = masks[slot];
                const int n = (int)min((int64_t)TT, len - (int64_t)k * TT);
                const unsigned char* ks = smem + slot * stage_bytes + local_head * D * esize;
                const unsigned char* vs = ks + TT * row_bytes;
                for (int sub = 0; sub < TT; sub += S::SC) {
                    float s[kTokensPerGroup][kItemHeads];
                    bool ok[kTokensPerGroup];
#pragma unroll
                    for (int i = 0; i < kTokensPerGroup; ++i) {
                        const int j = sub + i * S::TPI + g;
                        ok[i] = j < n && ((mask >> j) & 1ull);
                        float dot[kItemHeads];
#pragma unroll
                        for (int h = 0; h < kItemHeads; ++h) dot[h] = 0.f;
                        if (ok[i]) {
                            const uint4* row = reinterpret_cast<const uint4*>(ks + j * row_bytes);
#pragma unroll
                            for (int v = 0; v < S::VPL; ++v) {
                                float f[S::E];
                                Elem<T>::load(row[lj + v * S::LPT], f);
#pragma unroll
                                for (int h = 0; h < kItemHeads; ++h)
#pragma unroll
                                    for (int e = 0; e < S::E; ++e) dot[h] = fmaf(qf[h][v][e], f[e], dot[h]);
                            }
                        }
#pragma unroll
                        for (int off = 1; off < S::LPT; off <<= 1)
#pragma unroll
                            for (int h = 0; h < kItemHeads; ++h)
                                dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], off);
#pragma unroll
                        for (int h = 0; h < kItemHeads; ++h) s[i][h] = ok[i] ? dot[h] * p.scale_log2 : -INFINITY;
                    }
                    float pr[kTokensPerGroup][kItemHeads];
#pragma unroll
                    for (int h = 0; h < kItemHeads; ++h) {
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
                        const uint4* row = reinterpret_cast<const uint4*>(vs + j * row_bytes);
#pragma unroll
                        for (int v = 0; v < S::VPL; ++v) {
                            float f[S::E];
                            Elem<T>::load(row[lj + v * S::LPT], f);
#pragma unroll
                            for (int h = 0; h < kItemHeads; ++h)
#pragma unroll
                                for (int e = 0; e < S::E; ++e) acc[h][v][e] = fmaf(pr[i][h], f[e], acc[h][v][e]);
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }
        if (active) {
            // Merge the lane groups (each saw every TPI-th token), then write.
            const bool final_row = cta_of_tile(prefix[b], G, total) == cta_of_tile(prefix[b + 1] - 1, G, total);
            const int record = b + c;
#pragma unroll
            for (int h = 0; h < kItemHeads; ++h) {
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
                if (g == 0 && h < item_heads) {
                    const int qh = kvh * p.group + chunk * kItemHeads + h;
                    if (final_row) {
                        uint4* orow = reinterpret_cast<uint4*>(static_cast<T*>(p.out) + ((int64_t)b * p.q_heads + qh) * D);
#pragma unroll
                        for (int v = 0; v < S::VPL; ++v) orow[lj + v * S::LPT] = Elem<T>::store(acc[h][v]);
                    } else {
                        float4* prow = reinterpret_cast<float4*>(p.partial + ((int64_t)record * p.q_heads + qh) * D);
#pragma unroll
                        for (int v = 0; v < S::VPL; ++v)
#pragma unroll
                            for (int e = 0; e < S::E; e += 4)
                                prow[((lj + v * S::LPT) * S::E + e) / 4] =
                                    make_float4(acc[h][v][e], acc[h][v][e + 1], acc[h][v][e + 2], acc[h][v][e + 3]);
                        if (lj == 0)
                            p.lse[(int64_t)record * p.q_heads + qh] = (L > 0.f) ? mx + log2f(L) : -INFINITY;
                    }
                }
            }
        }
        t = seg_hi;
    }
}

// Merge the partial records of every request that spans several CTAs; write
// zero rows for requests with no tiles (invalid length).  One warp per
// (request, query head).
template <typename T>
__global__ void __launch_bounds__(256) paged_decode_combine_kernel(const DecodeParams p, int D, int G) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= p.batch * p.q_heads) return;
    const int b = row / p.q_heads, qh = row % p.q_heads;
    const int* prefix = p.prefix_out;
    const int total = prefix[p.batch];
    const int t0 = prefix[b], t1 = prefix[b + 1];
    T* out = static_cast<T*>(p.out) + (int64_t)row * D;
    if (t1 == t0) {
        for (int d = lane; d < D; d += 32) out[d] = Elem<T>::from_float(0.f);
        return;
    }
    const int c0 = cta_of_tile(t0, G, total), c1 = cta_of_tile(t1 - 1, G, total);
    if (c0 == c1) return;  // a single CTA wrote the final row
    const int n = c1 - c0 + 1;
    const int64_t first = (int64_t)b + c0;
    // CTAs whose tile range is empty (grid larger than the batch's tile count)
    // wrote no record: their weight is zero.
    auto owns_tiles = [&](int k) {
        const int64_t cta = c0 + k;
        return (cta * total) / G != ((cta + 1) * total) / G;
    };
    float mx = -INFINITY;
    for (int k = lane; k < n; k += 32)
        if (owns_tiles(k)) mx = fmaxf(mx, p.lse[(first + k) * p.q_heads + qh]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    constexpr int kMaxDimsPerLane = 8;  // D <= 256
    float acc[kMaxDimsPerLane];
#pragma unroll
    for (int i = 0; i < kMaxDimsPerLane; ++i) acc[i] = 0.f;
    float wsum = 0.f;
    for (int base = 0; base < n; base += 32) {
        float w = 0.f;
        if (base + lane < n && mx != -INFINITY && owns_tiles(base + lane)) {
            const float lse = p.lse[(first + base + lane) * p.q_heads + qh];
            w = (lse == -INFINITY) ? 0.f : exp2f(lse - mx);
        }
        const int count = min(32, n - base);
        for (int k = 0; k < count; ++k) {
            const float wk = __shfl_sync(0xffffffffu, w, k);
            wsum += wk;
            if (wk == 0.f) continue;
            const float* part = p.partial + ((first + base + k) * p.q_heads + qh) * D;
#pragma unroll
            for (int i = 0; i < kMaxDimsPerLane; ++i) {
                const int d = lane + 32 * i;
                if (d < D) acc[i] = fmaf(wk, part[d], acc[i]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kMaxDimsPerLane; ++i) {
        const int d = lane + 32 * i;
        if (d < D) out[d] = Elem<T>::from_float(wsum > 0.f ? acc[i] / wsum : 0.f);
    }
}

}  // namespace minikv

#include "decode_mma.cu"

namespace minikv {

// ------------------------------------------------------------------ host side
struct DecodePlan {
    bool mma;
    int tile_tokens, stages, row_bytes, heads_per_cta, chunks_per_head, chunk_groups, head_groups;
    int grid, smem_bytes;
    int64_t records, ws_prefix, ws_lse, ws_partial, ws_bytes;
};

static int esize_of(int dtype) { return dtype == 0 ? 4 : 2; }

static int lanes_per_token(int D, int esize) {
    const int vr = D * esize / 16;
    return (vr % 8 == 0) ? 8 : (vr % 4 == 0) ? 4 : 2;
}

static int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

// Everything here depends on shapes and the device only (graph-static).
// fp16/bf16 use the tensor-core consumer (decode_mma.cu): warps own up to 16
// query heads, shared-memory rows are padded by 16 bytes and tiles are
// multiples of 16 tokens.  fp32 uses the CUDA-core consumer above.
static bool make_decode_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t D, int64_t block_size,
                             int64_t table_width, int dtype, int sm_count, DecodePlan* plan) {
    const int es = esize_of(dtype);
    const bool mma = dtype != 0;
    const int sc = mma ? 16 : kTokensPerGroup * (32 / lanes_per_token((int)D, es));
    const int heads_per_item = mma ? 16 : kItemHeads;
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
    const int row = hpc * (int)D * es + (mma ? 16 : 0);  // shared-memory row stride
    int tt = (32768 / row) / sc * sc;
    tt = std::max(sc, std::min(64, tt));
    const int stage = 2 * tt * row;
    const int fixed = (int)((B + 1) * 4) + 128;
    const int max_smem = 232448 - 1024;  // opt-in limit per block, minus static smem
    int stages = std::min(4, (196608 + 4096) / stage);
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
    plan->row_bytes = row;
    plan->heads_per_cta = hpc;
    plan->chunks_per_head = cph;
    plan->chunk_groups = ncg;
    plan->head_groups = z;
    plan->grid = (int)grid;
    plan->smem_bytes = smem;
    plan->records = B + grid - 1;
    plan->ws_prefix = 0;
    plan->ws_lse = align256((B + 1) * 4);
    plan->ws_partial = plan->ws_lse + align256(plan->records * Hq * 4);
    plan->ws_bytes = plan->ws_partial + align256(plan->records * Hq * D * 4);
    return true;
}

template <typename Kernel>
static cudaError_t set_smem(Kernel kernel, int bytes) {
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

template <typename T, int D>
static cudaError_t launch_decode_typed(const DecodeParams& p, const DecodePlan& plan, cudaStream_t stream) {
    cudaError_t err;
    if constexpr (sizeof(T) == 2) {
        auto kernel = paged_decode_mma_kernel<T, D>;
        err = set_smem(kernel, plan.smem_bytes);
        if (err != cudaSuccess) return err;
        kernel<<<dim3(plan.grid, plan.head_groups), kDecodeThreads, plan.smem_bytes, stream>>>(p);
    } else {
        auto kernel = paged_decode_split_kernel<T, D>;
        err = set_smem(kernel, plan.smem_bytes);
        if (err != cudaSuccess) return err;
        kernel<<<dim3(plan.grid, plan.head_groups), kDecodeThreads, plan.smem_bytes, stream>>>(p);
    }
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const int rows = p.batch * p.q_heads;
    paged_decode_combine_kernel<T><<<(rows + 7) / 8, 256, 0, stream>>>(p, D, plan.grid);
    return cudaGetLastError();
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

static int run_decode(const void* query, const void* key_cache, const void* value_cache,
                      const int64_t* block_tables, const int64_t* context_lens, const int64_t* table_rows,
                      void* out, void* workspace, int64_t workspace_bytes, int64_t batch, int64_t q_heads,
                      int64_t kv_heads, int64_t head_dim, int64_t num_blocks, int64_t block_size,
                      int64_t table_width, int dtype, cudaStream_t stream) {
    DecodePlan plan;
    if (!make_decode_plan(batch, q_heads, kv_heads, head_dim, block_size, table_width, dtype, sm_count(), &plan))
        return fail(MINIKV_EUNSUPPORTED, "decode shape does not fit shared memory (batch too large?)");
    MINIKV_REQUIRE(workspace != nullptr && workspace_bytes >= plan.ws_bytes && aligned16(workspace),
                   MINIKV_EINVAL, "decode workspace too small or misaligned");
    DecodeParams p{};
    p.q = query;
    p.kc = key_cache;
    p.vc = value_cache;
    p.tables = block_tables;
    p.lens = context_lens;
    p.table_rows = table_rows;
    p.out = out;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    p.prefix_out = reinterpret_cast<int*>(ws + plan.ws_prefix);
    p.lse = reinterpret_cast<float*>(ws + plan.ws_lse);
    p.partial = reinterpret_cast<float*>(ws + plan.ws_partial);
    p.batch = (int)batch;
    p.q_heads = (int)q_heads;
    p.kv_heads = (int)kv_heads;
    p.num_blocks = (int)std::min<int64_t>(num_blocks, 2147483647);
    p.block_size = (int)block_size;
    p.table_width = (int)table_width;
    p.group = (int)(q_heads / kv_heads);
    p.chunks_per_head = plan.chunks_per_head;
    p.heads_per_cta = plan.heads_per_cta;
    p.chunk_groups = plan.chunk_groups;
    p.tile_tokens = plan.tile_tokens;
    p.stages = plan.stages;
    p.row_bytes = plan.row_bytes;
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
    cudaError_t err = launch_decode(dtype, (int)head_dim, p, plan, stream);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_decode launch");
    return MINIKV_OK;
}

}  // namespace minikv
