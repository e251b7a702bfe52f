// Ragged causal paged prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Work item = one 128-row query tile of one request for one kv head: the rows
// are tm = 128 / group consecutive query tokens x the group's query heads
// (GQA packing, so every K/V tile is loaded once for all query heads that
// read it).  The grid is persistent (one CTA per SM): every CTA orders the
// query tiles by their number of key tiles, longest first (the same order in
// every CTA, computed from the device metadata), and takes items in
// boustrophedon order, so the long items start first and the CTAs end
// together.  TMEM, the barriers and the warp pipeline live across items: the
// next item's Q is loaded as soon as the last S MMA of the current item has
// read Q, and its first P V waits only until the epilogue has read O.  An
// item walks the request's key tiles of 128 keys, up to its last query
// position (causal):
//   S_j = Q K_j^T   tcgen05.mma kind::f16, M=128, N=128, K=D -> TMEM (fp32),
//                   double-buffered (two 128-column S buffers)
//   P_j = exp2(S_j * log2(e)/sqrt(D) - m)   (softmax warps), written as 16-bit
//                   values over the first 64 columns of S_j's own TMEM buffer
//   O  += P_j V_j   tcgen05.mma with A = P_j read from TMEM, M=128, N=D, K=128
//                   -> TMEM (fp32), accumulated across key tiles
// The running max m is raised lazily: while no score exceeds it by more than
// 8 (log2 units) P is formed against the old m, so O is rescaled in TMEM
// (tcgen05.ld / st by the row's thread) only when m moves by more than that.
// Warp roles: warps 0 and 10 issue the TMA loads (Q once; the K and V boxes of
// each key tile straight from the physical pages of the block table,
// SWIZZLE_128B; warp 0 runs the K ring and warp 10 the V ring, two slots each,
// each slot freed by the MMA that reads it) and warp 0 publishes each tile's
// key-validity bits; warp 1 owns the TMEM allocation and one of its lanes issues every MMA
// as soon as its operands are ready, so S runs up to two tiles ahead of P V
// and the scores of the next tile are computed while the softmax warps work;
// warps 2-9 are two softmax warpgroups: a row (= TMEM lane) has one thread in
// each, for half of its keys and half of O, so the P tile, the rescale and the
// epilogue are split two ways.  Because P stays in TMEM, the softmax of tile
// j+1 runs while P_j V_j is on the tensor cores.  No TMA multicast.
//
// FP8 pools (template F8 = 1 E4M3, 2 E5M2; head_dim 128): the K and V boxes
// carry one-byte codes (one 128-byte box per page and kv head instead of two),
// land in the second K-block of a ring slot and are converted in place to
// fp16 by the producer warp before it releases the slot; S and P V then run
// in fp16 (a bf16 query tile is converted to fp16 in shared memory once per
// item), with the pool's scales folded into the softmax scale and the output.
//
// Semantics follow the reference kernel (mini_engine/kernels/csrc/prefill.cu:
// 104-185): row t of request r attends keys [0, start_r + t]; keys on a page
// id outside [0, num_blocks) are masked; rows whose position falls outside
// the context or the table get zeros.  Keys past the context and keys of
// masked pages have their V rows zeroed in shared memory before the PV product.
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace minikv {

constexpr int kPfThreads = 352;  // warp 0 K loads, 1 MMA/TMEM, 2-9 softmax (two warpgroups), 10 V loads
constexpr int kPfVWarp = 10;
constexpr int kPfMaxRequests = 4096;  // requests of one launch on this route (query-tile prefix in smem)
constexpr int kPfMaxSort = 1024;      // query tiles sorted by cost; beyond that, natural order
constexpr int kPfRows = 128;     // M rows per CTA (tokens x GQA heads)
constexpr int kPfKeys = 128;     // keys per tile

struct PrefillTcParams {
    const int64_t* cu_q;
    const int64_t* starts;
    const int64_t* tables;
    const int64_t* ctx;
    void* out;
    int requests, q_heads, kv_heads, group, num_blocks, block_size, table_width;
    int tm;        // query tokens per tile = 128 / group
    int box_rows;  // rows per K/V TMA box (divides block_size and 128, >= 8)
    float scale_log2;
    float out_scale;  // multiplies the output (an FP8 pool's value scale; 1 otherwise)
};

// 2^x on the special-function unit (ex2.approx, flush to zero); 2^-inf = 0.
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Barrier of the 256 softmax threads (both warpgroups).
__device__ __forceinline__ void softmax_sync() {
    asm volatile("bar.sync 2, 256;" ::: "memory");
}

template <typename T, int D>
struct PfLayout {
    static constexpr int KB = D / 64;                     // 128-byte K-blocks per row
    static constexpr int Q_BYTES = kPfRows * D * 2;
    static constexpr int KV_BYTES = kPfKeys * D * 2;
    static constexpr int BLOCK_BYTES = 128 * 128;         // one K-block of a 128-row operand
    static constexpr int OFF_K = Q_BYTES;
    static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;
    static constexpr int OFF_BAR = OFF_V + 2 * KV_BYTES;
    static constexpr int OFF_RED = OFF_BAR + 512;          // [2][2][128] partial row maxima, [2][128] sums
    static constexpr int OFF_PFX = OFF_RED + 3 * 1024;      // [kPfMaxRequests + 1] query-tile prefix
    static constexpr int OFF_ORD = OFF_PFX + 4 * (kPfMaxRequests + 4);  // [kPfMaxSort] sorted query tiles
    static constexpr int SMEM = OFF_ORD + 8 * kPfMaxSort + 1024;        // + alignment slack
    static constexpr uint32_t TMEM_COLS = 512;  // S/P 0, S/P 1 (128 columns each) and O (D columns)
};

// Query tiles of the batch, for the persistent schedule: qt_pfx[r] = number of
// 128-row query tiles of requests < r.  One work item = (query tile, kv head).
struct PfItem {
    int r, m, h, n_tiles, qlen, t_lo;
    int64_t q0, start, limit;
    const int64_t* table;
};

// Key tiles (of 128 keys) the item's rows attend, causally: 0 for an empty item.
__device__ __forceinline__ int pf_item_tiles(const PrefillTcParams& p, int r, int m, int64_t* q0_out, int* qlen_out,
                                             int64_t* start_out, int64_t* limit_out) {
    const int64_t q0 = p.cu_q[r];
    const int qlen = (int)(p.cu_q[r + 1] - q0);
    const int64_t start = p.starts[r];
    const int64_t cap = (int64_t)p.table_width * p.block_size;
    const int64_t limit = min(p.ctx[r], cap);  // keys [0, limit) exist
    const int t_lo = m * p.tm;
    const int64_t p_last = min(start + min(t_lo + p.tm, qlen) - 1, limit - 1);
    if (q0_out) {
        *q0_out = q0;
        *qlen_out = qlen;
        *start_out = start;
        *limit_out = limit;
    }
    return (p_last < 0 || start < 0) ? 0 : (int)(p_last / kPfKeys + 1);
}

// Request owning natural query tile qt: largest r with qt_pfx[r] <= qt.
__device__ __forceinline__ int pf_request_of(const int* qt_pfx, int B, int qt) {
    int lo = 0, hi = B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (qt_pfx[mid] <= qt) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ PfItem pf_item(const PrefillTcParams& p, const int* qt_pfx, const uint32_t* order,
                                          bool sorted, int item, int kv_heads) {
    PfItem w;
    const int slot = item / kv_heads;
    const int qt = sorted ? (int)(order[slot] & 0xFFFFFu) : slot;
    w.h = item % kv_heads;
    w.r = pf_request_of(qt_pfx, p.requests, qt);
    w.m = qt - qt_pfx[w.r];
    w.t_lo = w.m * p.tm;
    w.n_tiles = pf_item_tiles(p, w.r, w.m, &w.q0, &w.qlen, &w.start, &w.limit);
    w.table = p.tables + (int64_t)w.r * p.table_width;
    return w;
}

// Item `k`-th of CTA c (boustrophedon over the cost-sorted items), or -1.
__device__ __forceinline__ int pf_nth_item(int k, int c, int G, int n_items) {
    const int i = k * G + ((k & 1) ? (G - 1 - c) : c);
    return i < n_items ? i : -1;
}

// FP8 pools (head_dim 128).  A key tile's codes (128 rows x 128 bytes, the
// TMA's 128-byte swizzle: chunk c of row r at 16-byte position c ^ (r & 7))
// land in the second K-block of a 16-bit ring slot; row r of that block is
// exactly the bytes of code row r.  A lane converts whole rows: it reads all
// eight chunks of row r, then writes dims 0..63 to row r of the first K-block
// and dims 64..127 over the codes it has read, so the conversion runs in place.
// E5M2 codes are the high bytes of their fp16 values; E4M3 codes are placed
// as fp16 of 2^-8 times their value (exact, subnormals included), and the
// factor 2^8 goes into the softmax scale (K) and the output scale (V).
template <int F8>
__device__ __forceinline__ void pf_convert_codes(unsigned char* slot, int lane) {
    constexpr int kBlock = 128 * 128;
#pragma unroll 1
    for (int r = lane; r < kPfKeys; r += 32) {
        const int sw = r & 7;
        const unsigned char* src = slot + kBlock + r * 128;
        uint4 in[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) in[c] = *reinterpret_cast<const uint4*>(src + ((c ^ sw) << 4));
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint32_t w[4] = {in[c].x, in[c].y, in[c].z, in[c].w};
            uint32_t h[8];  // dims 16c .. 16c + 15 as fp16 pairs
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t lo = byte_perm(w[i], 0u, 0x1404u), hi = byte_perm(w[i], 0u, 0x3424u);
                h[2 * i] = F8 == 1 ? e4m3x2_to_h2_scaled(lo) : lo;
                h[2 * i + 1] = F8 == 1 ? e4m3x2_to_h2_scaled(hi) : hi;
            }
            unsigned char* dst = slot + (c >> 2) * kBlock + r * 128;
            const int k0 = (2 * c) & 7;
            *reinterpret_cast<uint4*>(dst + ((k0 ^ sw) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
            *reinterpret_cast<uint4*>(dst + (((k0 + 1) ^ sw) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
        }
    }
}

// fp16 pair (saturated to the finite range) of a bf16 pair.
__device__ __forceinline__ uint32_t bf16x2_to_h2_sat(uint32_t w) {
    uint32_t h;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(h) : "f"(__uint_as_float(w & 0xffff0000u)),
        "f"(__uint_as_float(w << 16)));
    return h;
}

// Half `part` (0 or 1) of a bf16 query tile converted in place to fp16, for the
// fp16 MMAs over FP8 pools (the K and V producer warps take one half each).
__device__ __forceinline__ void pf_convert_q_bf16(unsigned char* sq, int bytes, int part, int lane) {
    uint4* q4 = reinterpret_cast<uint4*>(sq) + part * (bytes / 32);
#pragma unroll 4
    for (int i = lane; i < bytes / 32; i += 32) {
        const uint4 v = q4[i];
        q4[i] = make_uint4(bf16x2_to_h2_sat(v.x), bf16x2_to_h2_sat(v.y), bf16x2_to_h2_sat(v.z), bf16x2_to_h2_sat(v.w));
    }
}

template <typename T, int D, int F8 = 0>
__global__ void __launch_bounds__(kPfThreads, 1) paged_prefill_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const PrefillTcParams p) {
    using L = PfLayout<T, D>;
    constexpr bool kBf16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
    // F8 = 1 (E4M3) or 2 (E5M2): K/V come from an FP8 pool through pf_convert_codes, and
    // the MMAs run in fp16 (a bf16 query tile is converted once per item)
    static_assert(F8 == 0 || D == 128, "FP8 pages are staged for head_dim 128 only");
    using C = typename std::conditional<F8 != 0, __half, T>::type;  // MMA operand type
    constexpr bool kMmaBf16 = F8 == 0 && kBf16;
    constexpr bool kConvertQ = F8 != 0 && kBf16;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* sQ = smem;
    unsigned char* sK = smem + L::OFF_K;
    unsigned char* sV = smem + L::OFF_V;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
    uint64_t* q_full = bar + 0;    // Q of the CTA's current item landed
    uint64_t* k_full = bar + 1;    // [2] K of a key tile landed (+ its key_ok words)
    uint64_t* k_empty = bar + 3;   // [2] the S MMA is done with that K slot
    uint64_t* v_full = bar + 5;    // [2] V of a key tile landed
    uint64_t* v_empty = bar + 7;   // [2] the P V MMA is done with that V slot
    uint64_t* s_full = bar + 9;    // [2] S of a tile is in its TMEM buffer
    uint64_t* q_empty = bar + 11;  // the last S MMA of an item has read Q
    uint64_t* o_free = bar + 12;   // the epilogue of an item has read O
    uint64_t* p_full = bar + 13;   // P of the tile is in its TMEM buffer, O rescaled, masked V rows zeroed
    uint64_t* o_done = bar + 14;   // the P V product of the tile has been accumulated into O
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 15);
    int* info = reinterpret_cast<int*>(bar + 16);               // number of query tiles, sorted flag
    // [4][4] validity bits of key tile g (CTA-wide tile counter) in slot g % 4:
    // the producer rewrites a slot for tile g + 4 only after S(g + 2), which
    // needs the softmax of tile g to have read its S buffer (and these words)
    uint32_t* key_ok = reinterpret_cast<uint32_t*>(bar + 18);
    uint64_t* mma_drain = bar + 26;  // the issuer's last commit: every MMA it issued has completed
    // [2] by S buffer: the MMA thread has issued S of the tile (after acquiring its K slot and key_ok
    // words).  The softmax waits here, not on k_full: at an item boundary the first two S of the next
    // item need no P V, so the K ring can complete a slot's phase twice before the softmax warps,
    // still in the previous item's epilogue, reach that tile, and a parity wait two phases behind
    // never returns; S(g + 2) waits for the softmax of tile g, so this barrier stays within one phase.
    uint64_t* bits_full = bar + 29;
    uint64_t* k8_full = bar + 32;  // [2] FP8 pools: the codes of a K tile landed (k_full: converted)
    uint64_t* v8_full = bar + 34;  // [2] the same for V
    uint64_t* q_ready = bar + 36;  // FP8 pools, bf16 query: both halves of Q converted to fp16
    int* qt_pfx = reinterpret_cast<int*>(smem + L::OFF_PFX);         // [requests + 1]
    uint32_t* order = reinterpret_cast<uint32_t*>(smem + L::OFF_ORD);  // [kPfMaxSort] sorted keys, then the keys

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int B = p.requests, G = p.group, TM = p.tm;
    // Chained launch: the metadata, q and the K/V pages may come from the previous kernel
    // (the slot scatter of the same step); the launch itself overlaps that kernel's tail.
    griddep_wait();
    griddep_launch_dependents();
    const int Hkv = p.kv_heads;

    // ---- query-tile prefix over the requests (warp 0)
    if (warp == 0) {
        int run = 0;
        for (int base = 0; base < B; base += 32) {
            const int r = base + lane;
            int t = 0;
            if (r < B) t = (int)((p.cu_q[r + 1] - p.cu_q[r] + TM - 1) / TM);
            if (t < 0) t = 0;
            int incl = t;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += v;
            }
            if (r < B) qt_pfx[r] = run + incl - t;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) {
            qt_pfx[B] = run;
            info[0] = run;
            info[1] = run <= kPfMaxSort ? 1 : 0;
        }
    }
    if (tid == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(o_free, 8);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1);
        }
        mbar_init(p_full, 8);
        mbar_init(o_done, 1);
        mbar_init(mma_drain, 1);
        mbar_init(&bits_full[0], 1);
        mbar_init(&bits_full[1], 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k8_full[s], 1);
            mbar_init(&v8_full[s], 1);
        }
        mbar_init(q_ready, 2);  // the two producer warps, one half of Q each
        mbar_init_fence();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_addr(tmem_slot)), "r"(L::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // columns: S0 [0,128) | S1 [128,256) | O [256, 256+D)
    const int n_qt = info[0];
    const bool sorted = info[1] != 0;
    const int n_items = n_qt * Hkv;

    // ---- longest first: order the query tiles by key tiles (descending), ties by
    // index, identically in every CTA.  Keys are unique, so a key's rank is the
    // number of smaller keys: two barriers, O(n^2 / threads) compares.
    if (sorted) {
        uint32_t* keys = order + kPfMaxSort;
        for (int i = tid; i < n_qt; i += blockDim.x) {
            const int r = pf_request_of(qt_pfx, B, i);
            const int cost = min(pf_item_tiles(p, r, i - qt_pfx[r], nullptr, nullptr, nullptr, nullptr), 1023);
            keys[i] = ((uint32_t)(1023 - cost) << 20) | (uint32_t)i;
        }
        __syncthreads();
        for (int i = tid; i < n_qt; i += blockDim.x) {
            const uint32_t key = keys[i];
            int rank = 0;
            for (int j = 0; j < n_qt; ++j) rank += keys[j] < key ? 1 : 0;
            order[rank] = key;
        }
        __syncthreads();
    }
    const int c = blockIdx.x, nC = gridDim.x;

    if (warp == 0 || warp == kPfVWarp) {
        if constexpr (F8 != 0) {
            // -------------------------------------------------------- FP8 producers
            // As below, with a tile's codes (one box of R rows x 128 bytes per page)
            // landing on k8_full / v8_full; the warp converts tile g after issuing the
            // loads of tile g + 1, then releases k_full / v_full.  The K warp converts
            // the last tile of an item before it waits to replace Q (the item's last S
            // needs it).  A bf16 Q is converted by both warps (one half each) after the
            // loads of the item's first key tile; the V warp's wait on Q's landing
            // cannot run ahead of the K warp's, as the V warp's first tile of item i + 1
            // waits for P V of item i, which needs the S of item i (and so its Q).
            const bool is_v = warp == kPfVWarp;
            const int box = lane;
            const unsigned full_mask = 0xffffffffu;
            const int R = p.box_rows, groups = kPfKeys / R;
            uint64_t* full = is_v ? v_full : k_full;
            uint64_t* land = is_v ? v8_full : k8_full;
            uint64_t* empty = is_v ? v_empty : k_empty;
            const CUtensorMap* map = is_v ? &tm_v : &tm_k;
            unsigned char* ring = is_v ? sV : sK;
            const uint64_t space_limit = space_wait_limit();
            int gt = 0, active = 0, pending = -1;
            bool stopped = false;
            auto convert = [&](int g) {
                const int slot = g & 1;
                // a landing that timed out (status bit set) is not read; the arrival still happens
                if (__all_sync(full_mask, mbar_wait(&land[slot], (g >> 1) & 1)))
                    pf_convert_codes<F8>(ring + slot * L::KV_BYTES, lane);
                fence_async_smem();
                tc_fence_before();
                __syncwarp(full_mask);
                if (lane == 0) mbar_arrive(&full[slot]);
            };
            for (int k = 0; !stopped; ++k) {
                const int it = pf_nth_item(k, c, nC, n_items);
                if (it < 0) break;
                const PfItem w = pf_item(p, qt_pfx, order, sorted, it, Hkv);
                if (w.n_tiles == 0) continue;
                if (!is_v) {
                    if (pending >= 0) {
                        convert(pending);
                        pending = -1;
                    }
                    int q_ok = 1;
                    if (lane == 0) {
                        if (active > 0) q_ok = mbar_wait_space(q_empty, (active - 1) & 1, space_limit) ? 1 : 0;
                        if (q_ok) {
                            mbar_arrive_expect_tx(q_full, (uint32_t)L::Q_BYTES);
#pragma unroll
                            for (int kb = 0; kb < L::KB; ++kb)
                                tma_load_3d(sQ + kb * L::BLOCK_BYTES, &tm_q, kb * 64, w.h * G, (int)(w.q0 + w.t_lo),
                                            q_full);
                        }
                    }
                    if (!__shfl_sync(full_mask, q_ok, 0)) break;
                }
                auto raw_page = [&](int j) -> int64_t {
                    const int64_t k0 = (int64_t)j * kPfKeys + box * R;
                    if (box >= groups || j >= w.n_tiles || k0 >= w.limit) return -1;
                    return w.table[k0 / p.block_size];
                };
                auto checked = [&](int64_t page) -> int64_t {
                    return (page >= 0 && page < p.num_blocks) ? page : -1;
                };
                int64_t page = checked(raw_page(0));
                int64_t next_raw = raw_page(1);
                for (int j = 0; j < w.n_tiles; ++j, ++gt) {
                    const int slot = gt & 1;
                    const int64_t key0 = (int64_t)j * kPfKeys;
                    const bool valid = page >= 0;
                    uint32_t words[4] = {0u, 0u, 0u, 0u};
                    if (!is_v) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint32_t bits = 0;
                            if (valid) {
                                const int64_t lo = max((int64_t)q * 32, (int64_t)box * R);
                                const int64_t hi =
                                    min(min((int64_t)q * 32 + 32, (int64_t)box * R + R), w.limit - key0);
                                if (hi > lo) {
                                    const int n = (int)(hi - lo);
                                    bits = (n == 32 ? 0xffffffffu : ((1u << n) - 1u)) << (int)(lo - q * 32);
                                }
                            }
                            words[q] = __reduce_or_sync(full_mask, bits);
                        }
                    }
                    const uint32_t bytes = (uint32_t)__popc(__ballot_sync(full_mask, valid)) * R * 128;
                    if (gt >= 2 &&
                        !__all_sync(full_mask, mbar_wait_space(&empty[slot], ((gt >> 1) - 1) & 1, space_limit))) {
                        stopped = true;
                        break;
                    }
                    if (box == 0) {
                        if (!is_v) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) key_ok[4 * (gt & 3) + q] = words[q];
                        }
                        mbar_arrive_expect_tx(&land[slot], bytes);
                    }
                    __syncwarp(full_mask);
                    if (valid) {
                        const int z = (int)(page * p.block_size + (key0 + box * R) % p.block_size);
                        tma_load_3d(ring + slot * L::KV_BYTES + L::BLOCK_BYTES + box * R * 128, map, 0, w.h, z,
                                    &land[slot]);
                    }
                    // (the V warp's previous tile first: the previous item's last P V needs it,
                    // and this item's Q may land much later)
                    if (pending >= 0) convert(pending);
                    pending = gt;
                    if (kConvertQ && j == 0) {
                        if (__all_sync(full_mask, mbar_wait(q_full, active & 1)))
                            pf_convert_q_bf16(sQ, L::Q_BYTES, is_v ? 1 : 0, lane);
                        fence_async_smem();
                        tc_fence_before();
                        __syncwarp(full_mask);
                        if (lane == 0) mbar_arrive(q_ready);
                    }
                    page = checked(next_raw);
                    next_raw = raw_page(j + 2);
                }
                ++active;
            }
            if (!stopped && pending >= 0) convert(pending);
            // Drain: every code tile issued (and Q) has landed before this warp exits.
            if (lane == 0) {
                for (int s2 = 0; s2 < 2 && s2 < gt; ++s2) mbar_drain(&land[s2], ((s2 + 2 * ((gt - 1 - s2) / 2)) >> 1) & 1);
                if (!is_v && active > 0) mbar_drain(q_full, (active - 1) & 1);
            }
            __syncwarp();
        } else {
            // -------------------------------------------------------- TMA producers
            // Warp 0 loads Q and K, warp 10 loads V, each on its own ring of two
            // slots, so a K slot is refilled as soon as the S MMA has read it,
            // whatever the P V MMAs are doing (two warps, because a warp that ran
            // both rings would reconverge after every wait).  Lane l owns box l
            // (R keys on one page) of a tile; its page id is read one tile ahead.
            const bool is_v = warp == kPfVWarp;
            const int box = lane;
            const unsigned full_mask = 0xffffffffu;
            const int R = p.box_rows, groups = kPfKeys / R;  // groups <= 16
            uint64_t* full = is_v ? v_full : k_full;
            uint64_t* empty = is_v ? v_empty : k_empty;
            const CUtensorMap* map = is_v ? &tm_v : &tm_k;
            unsigned char* ring = is_v ? sV : sK;
            const uint64_t space_limit = space_wait_limit();
            int gt = 0, active = 0;  // key tiles issued, items whose Q was issued
            bool stopped = false;    // a space wait gave up: issue nothing more, drain, exit
            for (int k = 0; !stopped; ++k) {
                const int it = pf_nth_item(k, c, nC, n_items);
                if (it < 0) break;
                const PfItem w = pf_item(p, qt_pfx, order, sorted, it, Hkv);
                if (w.n_tiles == 0) continue;
                if (!is_v) {
                    int q_ok = 1;
                    if (lane == 0) {
                        if (active > 0) q_ok = mbar_wait_space(q_empty, (active - 1) & 1, space_limit) ? 1 : 0;
                        if (q_ok) {
                            mbar_arrive_expect_tx(q_full, (uint32_t)L::Q_BYTES);
#pragma unroll
                            for (int kb = 0; kb < L::KB; ++kb)
                                tma_load_3d(sQ + kb * L::BLOCK_BYTES, &tm_q, kb * 64, w.h * G, (int)(w.q0 + w.t_lo),
                                            q_full);
                        }
                    }
                    if (!__shfl_sync(full_mask, q_ok, 0)) break;
                }
                // Page-table entry of this lane's box of tile j (-1: no box).  The entry of
                // tile j + 2 is loaded while tile j is issued and checked an iteration
                // later, so the table load never stalls the issue of a tile.
                auto raw_page = [&](int j) -> int64_t {
                    const int64_t k0 = (int64_t)j * kPfKeys + box * R;
                    if (box >= groups || j >= w.n_tiles || k0 >= w.limit) return -1;
                    return w.table[k0 / p.block_size];
                };
                auto checked = [&](int64_t page) -> int64_t {
                    return (page >= 0 && page < p.num_blocks) ? page : -1;
                };
                int64_t page = checked(raw_page(0));
                int64_t next_raw = raw_page(1);
                for (int j = 0; j < w.n_tiles; ++j, ++gt) {
                    const int slot = gt & 1;
                    const int64_t key0 = (int64_t)j * kPfKeys;
                    const bool valid = page >= 0;
                    uint32_t words[4] = {0u, 0u, 0u, 0u};
                    if (!is_v) {
                        // validity bits of the tile's keys: a key is valid when its box is and it is < limit
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            uint32_t bits = 0;
                            if (valid) {
                                const int64_t lo = max((int64_t)q * 32, (int64_t)box * R);
                                const int64_t hi = min(min((int64_t)q * 32 + 32, (int64_t)box * R + R), w.limit - key0);
                                if (hi > lo) {
                                    const int n = (int)(hi - lo);
                                    bits = (n == 32 ? 0xffffffffu : ((1u << n) - 1u)) << (int)(lo - q * 32);
                                }
                            }
                            words[q] = __reduce_or_sync(full_mask, bits);
                        }
                    }
                    const uint32_t bytes = (uint32_t)__popc(__ballot_sync(full_mask, valid)) * L::KB * R * 128;
                    if (gt >= 2 && !__all_sync(full_mask, mbar_wait_space(&empty[slot], ((gt >> 1) - 1) & 1, space_limit))) {
                        stopped = true;  // the MMAs may still read this slot
                        break;
                    }
                    if (box == 0) {
                        if (!is_v) {
#pragma unroll
                            for (int q = 0; q < 4; ++q) key_ok[4 * (gt & 3) + q] = words[q];
                        }
                        mbar_arrive_expect_tx(&full[slot], bytes);
                    }
                    __syncwarp(full_mask);
                    if (valid) {
                        const int z = (int)(page * p.block_size + (key0 + box * R) % p.block_size);
                        unsigned char* dst = ring + slot * L::KV_BYTES + box * R * 128;
#pragma unroll
                        for (int kb = 0; kb < L::KB; ++kb)
                            tma_load_3d(dst + kb * L::BLOCK_BYTES, map, kb * 64, w.h, z, &full[slot]);
                    }
                    page = checked(next_raw);
                    next_raw = raw_page(j + 2);
                }
                ++active;
            }
            // Drain: the last phase issued into each slot (and Q's) has landed before this
            // warp exits, so no TMA copy is in flight when the CTA releases its shared memory.
            if (lane == 0) {
                for (int s2 = 0; s2 < 2 && s2 < gt; ++s2) mbar_drain(&full[s2], ((s2 + 2 * ((gt - 1 - s2) / 2)) >> 1) & 1);
                if (!is_v && active > 0) mbar_drain(q_full, (active - 1) & 1);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // S(j) and P V(j) are issued in whichever order their operands become
        // ready (non-blocking probes), so a late K tile never holds back a
        // P V product whose P is done, and S runs up to two tiles ahead.
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc(128, kPfKeys, kMmaBf16, false);
            constexpr uint32_t idesc_o = umma_idesc(128, D, kMmaBf16, true);
            const uint32_t t_o = tmem + 2 * kPfKeys;
            const uint32_t q_addr = smem_addr(sQ);
            int gt = 0, active = 0;
            bool failed = false;
            for (int k = 0; !failed; ++k) {
                const int it = pf_nth_item(k, c, nC, n_items);
                if (it < 0) break;
                const PfItem w = pf_item(p, qt_pfx, order, sorted, it, Hkv);
                const int n_tiles = w.n_tiles;
                if (n_tiles == 0) continue;
                mbar_wait(kConvertQ ? q_ready : q_full, active & 1);
                int ns = 0, npv = 0;  // next S and next P V of this item
                uint64_t idle_since = 0;
                while (npv < n_tiles) {
                    bool progressed = false;
                    if (ns < n_tiles) {
                        const int gs = gt + ns, slot = gs & 1;
                        // the buffer of S(gs) holds P(gs - 2) until P V(gs - 2) has read it: MMAs of
                        // one thread run in issue order, so S(gs) goes after that product is issued
                        // (for the first two tiles of an item, every earlier product is issued)
                        if ((ns < 2 || npv >= ns - 1) && mbar_test_wait(&k_full[slot], (gs >> 1) & 1)) {
                            tc_fence_after();
                            const uint32_t k_addr = smem_addr(sK + slot * L::KV_BYTES);
#pragma unroll
                            for (int kk = 0; kk < D / 16; ++kk) {
                                const uint32_t off = (kk >> 2) * L::BLOCK_BYTES + (kk & 3) * 32;
                                umma_f16(tmem + slot * kPfKeys, smem_desc(q_addr + off, 16, 1024),
                                         smem_desc(k_addr + off, 16, 1024), idesc_s, kk > 0);
                            }
                            umma_commit(&s_full[slot]);
                            umma_commit(&k_empty[slot]);
                            mbar_arrive(&bits_full[slot]);  // release: the key_ok words acquired with K
                            if (ns == n_tiles - 1) umma_commit(q_empty);
                            ++ns;
                            progressed = true;
                        }
                    }
                    const int gp = gt + npv;
                    if (npv < ns && (npv > 0 || active == 0 || mbar_test_wait(o_free, (active - 1) & 1)) &&
                        mbar_test_wait(&v_full[gp & 1], (gp >> 1) & 1) && mbar_test_wait(p_full, gp & 1)) {
                        tc_fence_after();
                        const uint32_t v_addr = smem_addr(sV + (gp & 1) * L::KV_BYTES);
#pragma unroll
                        for (int kk = 0; kk < kPfKeys / 16; ++kk)  // P: 16 keys = 8 TMEM columns per step
                            umma_f16_tmem_a(t_o, tmem + (gp & 1) * kPfKeys + kk * 8,
                                            smem_desc(v_addr + kk * 16 * 128, L::BLOCK_BYTES, 1024), idesc_o,
                                            (npv > 0 || kk > 0));
                        umma_commit(o_done);
                        umma_commit(&v_empty[gp & 1]);
                        ++npv;
                        progressed = true;
                    }
                    if (progressed) {
                        idle_since = 0;
                    } else {
                        // bounded: the same limit as every other wait, then give up (status bit set)
                        __nanosleep(32);
                        const uint64_t now = global_ns();
                        if (idle_since == 0) {
                            idle_since = now;
                        } else if (now - idle_since > kWaitLimitNs ||
                                   (now - idle_since > kWaitCheckNs &&
                                    (*reinterpret_cast<volatile unsigned int*>(&g_status) & kStatusWaitTimeout))) {
                            raise_status(kStatusWaitTimeout);
                            failed = true;
                            break;
                        }
                    }
                }
                gt += n_tiles;
                ++active;
            }
            // every MMA issued above has completed before TMEM is released (and before
            // the shared-memory operands it reads go away)
            umma_commit(mma_drain);
            mbar_drain(mma_drain, 0);
        }
    } else {
        // ------------------------------------------------------------ softmax warps
        // Two warpgroups; the thread of warpgroup `half` for a row owns key
        // columns [64 half, 64 half + 64) of S and P and O columns
        // [half D/2, (half + 1) D/2).  The two threads of a row exchange their
        // partial maxima once per tile (shared memory + a 256-thread barrier),
        // keep partial sums, and add them at the end of the item.
        constexpr int kHalfKeys = kPfKeys / 2, kHalfD = D / 2;
        float* red = reinterpret_cast<float*>(smem + L::OFF_RED);  // [2][2][128] maxima, then [2][128] sums
        const int sw = warp - 2;                 // 0..7
        const int half = sw >> 2;                // warpgroup
        const int quarter = warp & 3;            // TMEM lane quarter of this warp
        const int row = quarter * 32 + lane;     // tile row = TMEM lane
        const int st = sw * 32 + lane;           // 0..255: masked-key V zeroing (row st & 127, K-blocks from st >> 7)
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        const uint32_t t_o = tmem + lane_base + 2 * kPfKeys + half * kHalfD;
        const float scale = p.scale_log2;
        int gt = 0;
        for (int k = 0;; ++k) {
            const int it = pf_nth_item(k, c, nC, n_items);
            if (it < 0) break;
            const PfItem w = pf_item(p, qt_pfx, order, sorted, it, Hkv);
            const int n_tiles = w.n_tiles;
            const int t = w.t_lo + row / G, g = row % G;
            const int64_t pos = w.start + t;
            const bool row_valid = t < w.qlen && pos < w.limit;
            // Running max (log2 domain) and partial sum.  The max is raised lazily: P
            // is computed against m_run as long as no score exceeds it by more than
            // 2^8, so O (accumulated in TMEM) is rescaled only when m_run moves.
            float m_run = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n_tiles; ++j) {
                const int gj = gt + j, slot = gj & 1;
                mbar_wait(&bits_full[slot], (gj >> 1) & 1);
                uint32_t wk[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) wk[q] = key_ok[4 * (gj & 3) + q];
                // keys [0, rel] of this tile are causally visible to the row
                const int64_t rel = pos - (int64_t)j * kPfKeys;
                uint32_t bits[2];
#pragma unroll
                for (int qq = 0; qq < 2; ++qq) {
                    const int q = 2 * half + qq;
                    const int64_t lim = rel - q * 32;
                    const uint32_t causal = lim >= 31 ? 0xffffffffu : (lim < 0 ? 0u : ((2u << (int)lim) - 1u));
                    bits[qq] = row_valid ? (wk[q] & causal) : 0u;
                }
                const bool full = (bits[0] & bits[1]) == 0xffffffffu;

                mbar_wait(&s_full[slot], (gj >> 1) & 1);
                tc_fence_after();
                float s[kHalfKeys];
                tmem_load_32(tmem + lane_base + slot * kPfKeys + half * kHalfKeys, s);
                tmem_load_32(tmem + lane_base + slot * kPfKeys + half * kHalfKeys + 32, s + 32);

                float mxs[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                if (full) {
#pragma unroll
                    for (int e = 0; e < kHalfKeys; ++e) mxs[e & 3] = fmaxf(mxs[e & 3], s[e]);
                } else {
#pragma unroll
                    for (int e = 0; e < kHalfKeys; ++e)
                        if ((bits[e >> 5] >> (e & 31)) & 1u) mxs[e & 3] = fmaxf(mxs[e & 3], s[e]);
                }
                float* mred = red + (gj & 1) * 256;
                mred[half * 128 + row] = fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3]));
                softmax_sync();  // also: both halves of the S buffer have been read, P may overwrite it
                const float mx = fmaxf(mred[row], mred[128 + row]);
                const float m_tile = mx * scale;  // -inf when the row sees no key of this tile
                float m_use = m_run, alpha = 1.f;
                bool rescale = false;
                if (m_tile > m_run + 8.f) {
                    alpha = (m_run == -INFINITY) ? 0.f : fast_exp2(m_run - m_tile);
                    rescale = m_run != -INFINITY;  // O holds only zeros while m_run is -inf
                    m_use = m_tile;
                }
                // P (16-bit, two keys per column) over the first 64 columns of this
                // tile's S buffer: keys 64 half .. 64 half + 63 at columns 32 half ..
                float sums[4] = {0.f, 0.f, 0.f, 0.f};
                const float neg = -m_use;
                float packed[32];
#pragma unroll
                for (int e = 0; e < kHalfKeys; e += 2) {
                    float pe[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int kx = e + u;
                        const float x = fast_exp2(fmaf(s[kx], scale, neg));
                        pe[u] = (full || ((bits[kx >> 5] >> (kx & 31)) & 1u)) ? x : 0.f;
                        sums[kx & 3] += pe[u];
                    }
                    packed[e / 2] = __uint_as_float(Elem<C>::pack(pe[0], pe[1]));
                }
                tmem_store_32(tmem + lane_base + slot * kPfKeys + half * 32, packed);
                tmem_store_wait();
                // O may be rescaled only once the previous P V product has landed in it
                if (j > 0) {
                    mbar_wait(o_done, (gj - 1) & 1);
                    tc_fence_after();
                }
                // tcgen05.ld / st are warp-wide (.sync.aligned): the whole warp takes
                // this branch when any of its rows rescales; the others scale by 1.
                if (__any_sync(0xffffffffu, rescale)) {
                    const float factor = rescale ? alpha : 1.f;
#pragma unroll
                    for (int cc = 0; cc < kHalfD / 32; ++cc) {
                        float v[32];
                        tmem_load_32(t_o + cc * 32, v);
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] *= factor;
                        tmem_store_32(t_o + cc * 32, v);
                    }
                    tmem_store_wait();
                }
                l_run = l_run * alpha + ((sums[0] + sums[1]) + (sums[2] + sums[3]));
                m_run = m_use;
                const int vrow_key = st & 127;
                if (!((wk[vrow_key >> 5] >> (vrow_key & 31)) & 1u) && mbar_wait(&v_full[slot], (gj >> 1) & 1)) {
                    // V rows of masked keys must be finite zeros before P V runs (a
                    // loaded box can hold rows past the context; unloaded rows hold stale data)
                    unsigned char* vrow = sV + slot * L::KV_BYTES + vrow_key * 128;
                    for (int kb = st >> 7; kb < L::KB; kb += 2) {
                        uint4* v4 = reinterpret_cast<uint4*>(vrow + kb * L::BLOCK_BYTES);
#pragma unroll
                        for (int cc = 0; cc < 8; ++cc) v4[cc] = make_uint4(0, 0, 0, 0);
                    }
                }
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full);
            }
            // row sum = the two threads' partial sums
            float* lred = red + 512;
            lred[half * 128 + row] = l_run;
            softmax_sync();
            const float l_row = lred[row] + lred[128 + row];
            if (n_tiles > 0) {
                mbar_wait(o_done, (gt + n_tiles - 1) & 1);
                tc_fence_after();
            }
            // every lane of the warp loads (warp-wide tcgen05.ld); rows past the chunk store nothing
            const float inv = (row_valid && l_row > 0.f) ? p.out_scale / l_row : 0.f;
            T* orow = static_cast<T*>(p.out) + ((w.q0 + t) * p.q_heads + w.h * G + g) * D + half * kHalfD;
#pragma unroll
            for (int cc = 0; cc < kHalfD / 32; ++cc) {
                float v[32];
                if (n_tiles > 0) {
                    tmem_load_32(t_o + cc * 32, v);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = 0.f;
                }
                if (t < w.qlen) {
#pragma unroll
                    for (int d = 0; d < 32; d += 8) {
                        float f[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) f[e] = v[d + e] * inv;
                        *reinterpret_cast<uint4*>(orow + cc * 32 + d) = Elem<T>::store(f);
                    }
                }
            }
            if (n_tiles > 0) {
                // O has been read: the next item's first P V may overwrite it
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(o_free);
            }
            softmax_sync();  // the sums of this item are read before the next item writes them
            gt += n_tiles;
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------------ host side
static int gcd_int(int a, int b) {
    while (b) {
        const int t = a % b;
        a = b;
        b = t;
    }
    return a;
}

// Shapes the tensor-core route handles.
static bool prefill_tc_supported(int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t block_size,
                                 int dtype, int64_t num_blocks, int64_t tokens, int64_t requests) {
    if (dtype == MINIKV_F32 || (head_dim != 64 && head_dim != 128)) return false;
    if (requests > kPfMaxRequests) return false;
    const int64_t group = q_heads / kv_heads;
    if (group < 1 || 128 % group != 0 || kv_heads > 65535) return false;
    if (gcd_int((int)std::min<int64_t>(block_size, 1 << 20), 128) < 8) return false;
    return num_blocks * block_size < (1ll << 31) && tokens < (1ll << 31) && encode_tiled_fn() != nullptr;
}

template <typename T, int D, int F8 = 0>
static cudaError_t launch_prefill_tc_typed(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                                           const PrefillTcParams& p, int grid, cudaStream_t stream) {
    using L = PfLayout<T, D>;
    auto kernel = paged_prefill_tc_kernel<T, D, F8>;
    static int configured[64] = {0};  // opt-in shared-memory size, set once per device
    cudaError_t err = ensure_smem_limit(kernel, L::SMEM, configured);
    if (err != cudaSuccess) return err;
    return launch_chained(kernel, dim3(grid), dim3(kPfThreads), (size_t)L::SMEM, stream, mq, mk, mv, p);
}

static int run_prefill_tc(const void* q, const void* key_cache, const void* value_cache, const int64_t* cu_seqlens_q,
                          const int64_t* query_starts, const int64_t* block_tables, const int64_t* context_lens,
                          void* out, int64_t tokens, int64_t requests, int64_t q_heads, int64_t kv_heads,
                          int64_t head_dim, int64_t num_blocks, int64_t block_size, int64_t table_width, int dtype,
                          cudaStream_t stream, double k_scale = 1.0, float v_scale = 1.f, int f8 = 0) {
    // f8: 0 = 16-bit pool; 1 / 2 = E4M3 / E5M2 pool (head_dim 128), codes converted in the kernel
    if (f8 != 0 && head_dim != 128) return fail(MINIKV_EINVAL, "FP8 pages are staged for head_dim 128 only");
    const bool bf16 = dtype == MINIKV_BF16;
    const int group = (int)(q_heads / kv_heads);
    const int tm = 128 / group;
    const int box_rows = gcd_int((int)std::min<int64_t>(block_size, 1 << 20), 128);
    CUtensorMap mq, mk, mv;
    if (!encode_map_3d(&mq, q, bf16, head_dim, q_heads, tokens, 64, group, tm) ||
        (f8 == 0 &&
         (!encode_map_3d(&mk, key_cache, bf16, head_dim, kv_heads, num_blocks * block_size, 64, 1, box_rows) ||
          !encode_map_3d(&mv, value_cache, bf16, head_dim, kv_heads, num_blocks * block_size, 64, 1, box_rows))) ||
        (f8 != 0 &&
         (!encode_map_3d_u8(&mk, key_cache, head_dim, kv_heads, num_blocks * block_size, 128, 1, box_rows) ||
          !encode_map_3d_u8(&mv, value_cache, head_dim, kv_heads, num_blocks * block_size, 128, 1, box_rows))))
        return fail(MINIKV_ECUDA, "cuTensorMapEncodeTiled failed for the paged prefill operands");
    PrefillTcParams p{};
    p.cu_q = cu_seqlens_q;
    p.starts = query_starts;
    p.tables = block_tables;
    p.ctx = context_lens;
    p.out = out;
    p.requests = (int)requests;
    p.q_heads = (int)q_heads;
    p.kv_heads = (int)kv_heads;
    p.group = group;
    p.num_blocks = (int)num_blocks;
    p.block_size = (int)block_size;
    p.table_width = (int)table_width;
    p.tm = tm;
    p.box_rows = box_rows;
    const double code_scale = f8 == 1 ? 256.0 : 1.0;  // E4M3 codes are converted to 2^-8 x their value
    p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim) * k_scale * code_scale);
    p.out_scale = (float)(v_scale * code_scale);
    // persistent grid: one CTA per SM, or fewer when the batch has fewer work items
    // (an upper bound: query tiles <= tokens / tm + requests, times the kv heads)
    const int64_t items_bound = ((tokens + tm - 1) / tm + requests) * kv_heads;
    if ((tokens + tm - 1) / tm + requests >= (1 << 20)) return fail(MINIKV_EINVAL, "too many paged prefill tiles");
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(items_bound, sm_count()));
    cudaError_t err;
    if (f8 != 0) {
        if (bf16)
            err = f8 == 1 ? launch_prefill_tc_typed<__nv_bfloat16, 128, 1>(mq, mk, mv, p, grid, stream)
                          : launch_prefill_tc_typed<__nv_bfloat16, 128, 2>(mq, mk, mv, p, grid, stream);
        else
            err = f8 == 1 ? launch_prefill_tc_typed<__half, 128, 1>(mq, mk, mv, p, grid, stream)
                          : launch_prefill_tc_typed<__half, 128, 2>(mq, mk, mv, p, grid, stream);
    } else if (bf16)
        err = head_dim == 64 ? launch_prefill_tc_typed<__nv_bfloat16, 64>(mq, mk, mv, p, grid, stream)
                             : launch_prefill_tc_typed<__nv_bfloat16, 128>(mq, mk, mv, p, grid, stream);
    else
        err = head_dim == 64 ? launch_prefill_tc_typed<__half, 64>(mq, mk, mv, p, grid, stream)
                             : launch_prefill_tc_typed<__half, 128>(mq, mk, mv, p, grid, stream);
    if (err != cudaSuccess) return cuda_fail(err, "minikv_paged_prefill tcgen05 launch");
    return MINIKV_OK;
}

}  // namespace minikv
