// Skinny projections of the batch decode step on the 5th-generation tensor
// cores (tcgen05 + TMEM, operands staged by TMA), with the element-wise steps
// around them fused in (mini_engine/model/native_qwen3.py:175-196 attention,
// :232-240 MLP, :260-277 layer; kernels/linear.py:116-130 the projections).
//
// Y[t, n] = sum_k X[t, k] W[n, k] for the decode batch (a few to a few hundred
// tokens t) and a weight W in nn.Linear layout [out_features, in_features].
// The weight is what streams from HBM, so it is the M side of the MMA (swap
// AB): a CTA computes D^T = W_tile X^T for a tile of 128 output features x NT
// tokens (NT <= 128; larger batches take several token chunks),
//   A = 128 weight rows x 64 in-features per k-block: one contiguous 16 KB
//       block of the packed weight (below), one 1-D bulk copy,
//   B = NT token rows x 64 in-features, cp.async by the math warps,
//   D = 128 TMEM lanes (features) x NT columns (tokens), fp32.
// The in-features are split over the S CTAs of a thread-block cluster
// (split-K, S <= 16).  CTA r owns a slice of the NT tokens: every CTA drains
// its fp32 partial tile from TMEM straight into the owners' shared memory
// (st.async, counted on the owner's mbarrier); the owner adds the S partials
// in rank order (the result does not depend on timing) and runs the fused
// epilogue on its tokens.
//
// Packed weights: the weight is stored once, at load time, as its shared-
// memory image: [tiles][k-blocks][128 rows][64 elements], each 8-row group
// with the 128B swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)) that
// the tensor core's SWIZZLE_128B K-major descriptor reads.  A row-major
// weight would need a TMA box of 128 separate 128-byte row segments per
// k-block, which the per-SM TMA unit fetches at a few ns per segment; a packed
// k-block is one contiguous bulk copy.  For the gate|up projection a tile
// holds 64 rows of gate and the matching 64 rows of up.
//
// Weights do not depend on earlier kernels: the producer issues the weight
// loads of the first ring slots before griddepcontrol.wait, so in a chained
// launch the weight stream overlaps the tail of the previous kernel, and only
// the X loads (and the epilogue's reads) wait for it.  The epilogue locates
// the KV slots while the MMAs run and reads its residual and rotary rows while
// the partial sums travel.
//
// Prologue (optional): RMSNorm of the X rows.  The per-row sums of squares
// come as partial sums over 128-feature tiles ([in_features / 128][tokens],
// written by the epilogue of the projection that produced X) and are added in
// tile order; the row is normalised in shared memory before the MMA reads it,
// rounded like the reference (T(T(x * rsqrt(mean + eps)) * w), fallback.py:8-10).
//
// Epilogues (every intermediate rounded to T at the reference's points):
//   kEpiStore     T(Y)
//   kEpiResidual  s = T(T(Y) + R) and the per-row partial sums of squares of s
//                 (o projection + residual add, down projection + residual add;
//                 elementwise.py:24-31)
//   kEpiSiluMul   a tile holds rows j of gate and rows j of up of the fused
//                 gate|up weight: T(T(silu(T(g))) * T(u))   (fallback.py:23-24)
//   kEpiQkRope    one tile = one head of the fused q|k|v projection (D = 128):
//                 q/k RMSNorm + rotary embedding (fallback.py:13-20), q written
//                 out, K and V appended to the paged pool with the guards of
//                 the decode KV append (data.cu:89-107)
//
// Warp roles: warp 0 issues the weight loads, warp 1 owns TMEM and one lane
// issues the MMAs, warps 2-3 prepare the epilogue's inputs, warps 4-7
// normalise X (prologue) and drain TMEM; all eight run the epilogue.  No TMA
// multicast.
#include <type_traits>

#include "common.cuh"
#include "tcgen05.cuh"

namespace minikv {

constexpr int kProjThreads = 256;
constexpr int kProjMaxStages = 8;
constexpr int kProjMaxSplit = 16;
constexpr int kProjMaxTokens = 128;     // NT: tokens per CTA
constexpr int kProjWBytes = 128 * 128;  // one k-block of the weight tile: 128 rows x 64 elements

enum { kEpiStore = 0, kEpiResidual = 1, kEpiSiluMul = 2, kEpiQkRope = 3 };

struct ProjParams {
    const void* w;     // packed weight: [tiles][k_blocks][128 x 64] (see above)
    const void* x;     // [tokens, in_features], rows x_stride elements apart
    int64_t x_stride;
    int tokens, in_features, out_features;
    int k_blocks;     // in_features / 64
    int split;        // S: CTAs of a cluster along the in-features (== gridDim.x)
    int tile_tokens;  // NT: tokens per CTA (multiple of 16, <= 128)
    int stages;       // ring slots
    int tmem_cols;
    int gate_offset;  // kEpiSiluMul: up rows = gate rows + gate_offset (the intermediate size)
    // prologue RMSNorm (ss_in == nullptr: none)
    const float* ss_in;  // [in_features / 128][tokens]
    const void* norm_weight;
    float eps;
    // epilogue
    void* out;
    int64_t out_stride;
    const void* residual;
    int64_t residual_stride;
    float* ss_out;  // kEpiResidual: [out_features / 128][tokens] (may be null)
    // kEpiQkRope
    const void* q_weight;
    const void* k_weight;
    const void* cos;  // [tokens, 64]
    const void* sin;
    void* key_cache;  // [num_blocks, block_size, kv_heads, 128]
    void* value_cache;
    const int64_t* tables;
    const int64_t* positions;
    int64_t width, num_blocks, block_size;
    int q_heads, kv_heads;
};

// Shared memory: [ring: stages x (W k-block | X k-block)] [recv: S x slice x 128 fp32]
// [inv: NT fp32] [kv slot per owned token: NT int64] [barriers]; the CTA's own
// fp32 partial tile ([NT][128]) is written over the drained ring.
struct ProjLayout {
    int stage_bytes, per, recv_slot, off_recv, off_inv, off_dst, off_bar, smem;
    __host__ __device__ ProjLayout(int nt, int stages, int split) {
        stage_bytes = kProjWBytes + nt * 128;
        per = (nt + split - 1) / split;  // tokens owned by each CTA of the cluster
        recv_slot = per * 512;
        int ring = stages * stage_bytes;
        if (ring < nt * 512) ring = nt * 512;
        off_recv = ring;
        off_inv = off_recv + (split > 1 ? split * recv_slot : 0);
        off_dst = off_inv + kProjMaxTokens * 4;
        off_bar = off_dst + kProjMaxTokens * 8;
        smem = off_bar + 256 + 1024;  // + alignment slack of the dynamic shared memory base
    }
};

__device__ __forceinline__ void proj_math_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Per-token inputs of the epilogue, read before the partial sums arrive.
struct ProjEpiIn {
    float a[4], b[4];  // residual (kEpiResidual) or cos / sin (kEpiQkRope) at the lane's features
};

template <typename T, int EPI>
__device__ __forceinline__ void proj_epilogue_inputs(const ProjParams& p, int tile, int64_t tok, int lane,
                                                     ProjEpiIn* in) {
    if (EPI == kEpiResidual) {
        Lane<T, 4>::load(static_cast<const T*>(p.residual) + tok * p.residual_stride + (int64_t)tile * 128 + lane * 4,
                         in->a);
    } else if (EPI == kEpiQkRope && tile < p.q_heads + p.kv_heads) {
        const int64_t angle = tok * 64 + (int64_t)(lane & 15) * 4;
        Lane<T, 4>::load(static_cast<const T*>(p.cos) + angle, in->a);
        Lane<T, 4>::load(static_cast<const T*>(p.sin) + angle, in->b);
    }
}

// Epilogue of one token row: lane l holds output features [4 l, 4 l + 4) of
// the tile; `dst` is the token's element offset in the KV pool for this tile's
// kv head and `w` the head's norm weights at those features (kEpiQkRope;
// dst -1: no append).
template <typename T, int EPI>
__device__ __forceinline__ void proj_epilogue(const ProjParams& p, int tile, int64_t tok, const float* acc,
                                              int64_t dst, const float* w, const ProjEpiIn& in, int lane) {
    if (EPI == kEpiStore) {
        T* out = static_cast<T*>(p.out) + tok * p.out_stride + (int64_t)tile * 128 + lane * 4;
        Lane<T, 4>::store(out, acc);
    } else if (EPI == kEpiResidual) {
        const int64_t col = (int64_t)tile * 128 + lane * 4;
        float y[4];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            y[j] = Narrow<T>::round(Narrow<T>::round(acc[j]) + in.a[j]);
            ss += y[j] * y[j];
        }
        Lane<T, 4>::store(static_cast<T*>(p.out) + tok * p.out_stride + col, y);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (p.ss_out != nullptr && lane == 0) p.ss_out[(int64_t)tile * p.tokens + tok] = ss;
    } else if (EPI == kEpiSiluMul) {
        // lanes 0-15: gate rows [64 tile + 4 l, +4); lanes 16-31: the matching up rows
        float y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float mine = Narrow<T>::round(acc[j]);
            const float up = __shfl_xor_sync(0xffffffffu, mine, 16);
            y[j] = Narrow<T>::round(mine / (1.0f + expf(-mine))) * up;
        }
        if (lane < 16)
            Lane<T, 4>::store(static_cast<T*>(p.out) + tok * p.out_stride + (int64_t)tile * 64 + lane * 4, y);
    } else {
        // kEpiQkRope: tile = head (q heads, then k heads, then v heads), head_dim 128
        const int h = tile;
        float x[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = Narrow<T>::round(acc[j]);
        if (h >= p.q_heads + p.kv_heads) {  // V: appended as projected
            if (dst >= 0) Lane<T, 4>::store(static_cast<T*>(p.value_cache) + dst + lane * 4, x);
            return;
        }
        const bool is_q = h < p.q_heads;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) ss += x[j] * x[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = rsqrtf(ss / 128.0f + p.eps);
#pragma unroll
        for (int j = 0; j < 4; ++j) x[j] = Narrow<T>::round(Narrow<T>::round(x[j] * inv) * w[j]);
        // rotary: first half  y1 = T(T(x1 c) - T(x2 s)); second half y2 = T(T(x1 s) + T(x2 c))
        const float* c = in.a;  // cos, sin at the lane's rotary angles
        const float* s = in.b;
        float y[4];
        const bool first = lane < 16;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float other = __shfl_xor_sync(0xffffffffu, x[j], 16);
            y[j] = first ? Narrow<T>::round(Narrow<T>::round(x[j] * c[j]) - Narrow<T>::round(other * s[j]))
                         : Narrow<T>::round(Narrow<T>::round(other * s[j]) + Narrow<T>::round(x[j] * c[j]));
        }
        if (is_q) {
            Lane<T, 4>::store(static_cast<T*>(p.out) + (tok * p.q_heads + h) * 128 + lane * 4, y);
        } else if (dst >= 0) {
            Lane<T, 4>::store(static_cast<T*>(p.key_cache) + dst + lane * 4, y);
        }
    }
}

// Element offset of token `tok`'s row for kv head `kvh` in the paged pool at
// its decode position, or -1 where the append is skipped (data.cu:89-107).
__device__ __forceinline__ int64_t proj_kv_slot(const ProjParams& p, int64_t tok, int kvh) {
    const int64_t logical = p.positions[tok];
    if (logical < 0) return -1;
    const int64_t index = logical / p.block_size;
    if (index >= p.width) return -1;
    const int64_t page = p.tables[tok * p.width + index];
    if (page < 0 || page >= p.num_blocks) return -1;
    return ((page * p.block_size + logical % p.block_size) * p.kv_heads + kvh) * 128;
}

// 16-byte copy global -> shared on the LSU path (zero-filled when !valid).
__device__ __forceinline__ void cp_async_16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 ::"r"(smem_addr(dst)), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed
// (the barrier's count includes these arrivals).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

template <typename T, int EPI, bool NORM>
__global__ void __launch_bounds__(kProjThreads, 1) proj_kernel(const ProjParams p) {
    constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NT = p.tile_tokens, STAGES = p.stages, S = p.split;
    const ProjLayout L(NT, STAGES, S);
    float* partial = reinterpret_cast<float*>(smem);  // [NT][128] fp32, over the drained ring
    float* recv = reinterpret_cast<float*>(smem + L.off_recv);  // [S][per tokens][128 features] fp32
    float* inv = reinterpret_cast<float*>(smem + L.off_inv);
    int64_t* kv_dst = reinterpret_cast<int64_t*>(smem + L.off_dst);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.off_bar);
    uint64_t* w_full = bar;          // [8] weight k-block landed (TMA)
    uint64_t* x_full = bar + 8;      // [8] X k-block landed (cp.async of the math warps)
    uint64_t* ready = bar + 16;      // [8] X k-block normalised and visible to the tensor core
    uint64_t* empty = bar + 24;      // [8] the MMAs are done with the slot
    uint64_t* acc_full = bar + 32;   // every MMA of the CTA has completed
    uint64_t* recv_full = bar + 33;  // the S partial slices of the owned tokens have landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 34);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // the cluster spans gridDim.x = S, so blockIdx.x is the CTA's rank in it
    const int rank = blockIdx.x, tile = blockIdx.y;
    const int tok0 = blockIdx.z * NT;
    const int kb0 = rank * p.k_blocks / S, nkb = (rank + 1) * p.k_blocks / S - kb0;
    const int t_lo = rank * L.per < NT ? rank * L.per : NT;
    const int t_hi = t_lo + L.per < NT ? t_lo + L.per : NT;  // owned tokens [t_lo, t_hi)
    const int pre = nkb < STAGES ? nkb : STAGES;
    float nw[4] = {1.f, 1.f, 1.f, 1.f};  // kEpiQkRope: this head's q_norm / k_norm weights (lane's features)
    if (EPI == kEpiQkRope && tile < p.q_heads + p.kv_heads)
        Lane<T, 4>::load(static_cast<const T*>(tile < p.q_heads ? p.q_weight : p.k_weight) + lane * 4, nw);

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&x_full[s], 128);
            mbar_init(&ready[s], 4);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(recv_full, 1);
        mbar_init_fence();
        if (S > 1 && t_hi > t_lo) mbar_arrive_expect_tx(recv_full, (uint32_t)(S * (t_hi - t_lo) * 512));
    }
    if (warp == 1) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (S > 1) cluster_arrive();  // this CTA's barriers are initialised (waited on before any remote store)
    const uint32_t tmem = *tmem_slot;
    griddep_launch_dependents();  // the next chained kernel may start streaming its weights

    if (warp == 0) {
        // ------------------------------------------------------------ weight producer (bulk copies)
        // weights do not depend on the previous kernel: no griddepcontrol.wait here
        if (lane == 0) {
            const uint64_t policy = policy_evict_first();  // streamed once per step
            const unsigned char* wsrc =
                static_cast<const unsigned char*>(p.w) + ((int64_t)tile * p.k_blocks + kb0) * kProjWBytes;
            for (int i = 0; i < nkb; ++i) {
                const int s = i % STAGES;
                if (i >= STAGES) mbar_wait(&empty[s], ((i / STAGES) - 1) & 1);
                mbar_arrive_expect_tx(&w_full[s], (uint32_t)kProjWBytes);
                bulk_load(smem + s * L.stage_bytes, wsrc + (int64_t)i * kProjWBytes, (uint32_t)kProjWBytes,
                          &w_full[s], policy);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = umma_idesc(128, NT, kBf16, false);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % STAGES;
                const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
                mbar_wait(&w_full[s], ph);
                mbar_wait(&ready[s], ph);
                tc_fence_after();
                const uint32_t a = smem_addr(smem + s * L.stage_bytes), b = a + kProjWBytes;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_f16(tmem, smem_desc(a + kk * 32, 16, 1024), smem_desc(b + kk * 32, 16, 1024), idesc,
                             (i > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(acc_full);
        }
        __syncwarp();
    } else if (warp < 4) {
        // ------------------------------------------------------------ epilogue inputs
        griddep_wait();
        const int e = tid - 64;  // 0..63
        for (int t = t_lo + e; t < t_hi; t += 64) {
            const int64_t tok = tok0 + t;
            if (tok >= p.tokens) break;
            if (EPI == kEpiQkRope) {
                const int h = tile;
                kv_dst[t] = h >= p.q_heads ? proj_kv_slot(p, tok, (h - p.q_heads) % p.kv_heads) : -1;
            }
        }
    } else {
        // ------------------------------------------------------------ math warps 4-7: X
        // Thread mt copies the 16-byte chunks q = mt + 128 n of each X k-block: row r = q / 8,
        // logical chunk q % 8 (= mt % 8 in every row), stored at chunk (q % 8) ^ (r % 8) of the
        // row (128B swizzle).  Rows past the batch are zero-filled.
        const int mt = tid - 128;
        const int lc = mt & 7, r_first = mt >> 3;
        const T* xg = static_cast<const T*>(p.x) + (int64_t)kb0 * 64 + lc * 8;
        const T* gamma = static_cast<const T*>(p.norm_weight) + (int64_t)kb0 * 64 + lc * 8;
        uint4 g_next = make_uint4(0, 0, 0, 0);
        if (NORM) g_next = ld_global_nc(gamma);  // weights: read before the wait
        griddep_wait();  // X (and its row statistics) come from the previous kernel
        auto issue = [&](int i) {
            unsigned char* xs = smem + (i % STAGES) * L.stage_bytes + kProjWBytes;
            for (int r = r_first; r < NT; r += 16) {
                const int tok = tok0 + r;
                const bool valid = tok < p.tokens;
                cp_async_16(xs + r * 128 + ((lc ^ (r & 7)) << 4),
                            xg + (int64_t)(valid ? tok : 0) * p.x_stride + (int64_t)i * 64, valid);
            }
            cp_async_arrive(&x_full[i % STAGES]);
        };
        for (int i = 0; i < pre; ++i) issue(i);
        if (NORM) {
            if (mt < NT) {
                const int tok = tok0 + mt;
                float f = 0.f;  // rows past the batch stay zero
                if (tok < p.tokens) {
                    const int tiles_in = p.in_features / 128;
                    const float* part = p.ss_in + tok;
                    float ss = 0.f;
                    int j = 0;
                    for (; j + 8 <= tiles_in; j += 8) {  // eight loads in flight, added in tile order
                        float v[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q) v[q] = part[(int64_t)(j + q) * p.tokens];
#pragma unroll
                        for (int q = 0; q < 8; ++q) ss += v[q];
                    }
                    for (; j < tiles_in; ++j) ss += part[(int64_t)j * p.tokens];
                    f = rsqrtf(ss / (float)p.in_features + p.eps);
                }
                inv[mt] = f;
            }
            proj_math_sync();
        }
        for (int i = 0; i < nkb; ++i) {
            const int s = i % STAGES;
            float w[8];
            if (NORM) {
                Elem<T>::load(g_next, w);
                if (i + 1 < nkb) g_next = ld_global_nc(gamma + (i + 1) * 64);
            }
            mbar_wait(&x_full[s], (uint32_t)(i / STAGES) & 1u);
            if (NORM) {
                unsigned char* xs = smem + s * L.stage_bytes + kProjWBytes;
                for (int r = r_first; r < NT; r += 16) {
                    uint4* ptr = reinterpret_cast<uint4*>(xs + r * 128 + ((lc ^ (r & 7)) << 4));
                    float x[8];
                    Elem<T>::load(*ptr, x);
                    const float f = inv[r];
#pragma unroll
                    for (int j = 0; j < 8; ++j) x[j] = Narrow<T>::round(x[j] * f) * w[j];
                    *ptr = Elem<T>::store(x);
                }
            }
            fence_async_smem();  // X in shared memory -> the MMA's async-proxy reads
            __syncwarp();
            if (lane == 0) mbar_arrive(&ready[s]);
            if (i + STAGES < nkb) {  // refill the slot once the MMAs of this k-block are done
                mbar_wait(&empty[s], (uint32_t)(i / STAGES) & 1u);
                issue(i + STAGES);
            }
        }
        // drain the accumulator: this warp may access TMEM lanes [32 (warp % 4), +32)
        mbar_wait(acc_full, 0);
        tc_fence_after();
        const int quad = warp & 3;
        const int f = quad * 32 + lane;
        for (int c0 = 0; c0 < NT; c0 += 16) {
            float v[16];
            tmem_load_16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
            for (int j = 0; j < 16; ++j) partial[(c0 + j) * 128 + f] = v[j];
        }
        tc_fence_before();
        if (S > 1) {
            // token t goes to owner o = t / per, row t - o per of the owner's slot for this rank:
            // 16 bytes per thread, one token row (512 contiguous bytes) per warp
            proj_math_sync();
            cluster_wait();  // every CTA of the cluster has initialised its barriers
            for (int q = mt; q < NT * 32; q += 128) {
                const int t = q >> 5, c = q & 31;
                const int o = t / L.per;
                const float* row = recv + (rank * L.per + (t - o * L.per)) * 128 + c * 4;
                st_async_f32<4>(cluster_addr(row, (uint32_t)o), partial + t * 128 + c * 4,
                                cluster_addr(recv_full, (uint32_t)o));
            }
        }
    }
    __syncthreads();  // partial tile (one CTA) and kv slots written; TMEM read
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
    }

    // ---------------------------------------------------------------- epilogue: warp w takes
    // tokens t_lo + w + 8 i; the first token's inputs are read while the partial sums arrive
    griddep_wait();  // (a no-op for the warps that waited already) the previous kernel's writes are visible
    int t = t_lo + warp;
    ProjEpiIn in{};
    if (t < t_hi && tok0 + t < p.tokens) proj_epilogue_inputs<T, EPI>(p, tile, tok0 + t, lane, &in);
    if (S > 1) {
        if (warp < 4) cluster_wait();  // (warps 4-7 passed it before their remote stores)
        if (t_hi > t_lo) mbar_wait(recv_full, 0);  // every CTA waits for what it is sent
    }
    for (; t < t_hi; t += kProjThreads / 32) {
        const int64_t tok = tok0 + t;
        if (tok >= p.tokens) break;
        if (t != t_lo + warp) proj_epilogue_inputs<T, EPI>(p, tile, tok, lane, &in);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const float* row = S == 1 ? partial + t * 128 + lane * 4 : recv + (t - t_lo) * 128 + lane * 4;
        const int rank_stride = L.per * 128;
        for (int r = 0; r < S; ++r) {  // rank order: the sum does not depend on timing
            const float4 v = *reinterpret_cast<const float4*>(row + r * rank_stride);
            acc[0] += v.x;
            acc[1] += v.y;
            acc[2] += v.z;
            acc[3] += v.w;
        }
        proj_epilogue<T, EPI>(p, tile, tok, acc, EPI == kEpiQkRope ? kv_dst[t] : -1, nw, in, lane);
    }
}

// Packed weight (see above) from a row-major [rows, in_features] weight: one
// thread per 16-byte chunk of the packed buffer.  pair_offset > 0: tile j
// holds rows [64 j, 64 j + 64) and [pair_offset + 64 j, ...) (gate | up).
template <typename T>
__global__ void __launch_bounds__(256) pack_linear_kernel(const T* __restrict__ w, T* __restrict__ packed,
                                                          int64_t chunks, int k_blocks, int64_t in_features,
                                                          int64_t pair_offset) {
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < chunks; q += (int64_t)gridDim.x * blockDim.x) {
        const int pc = (int)(q & 7), r = (int)((q >> 3) & 127);
        const int64_t block = q >> 10;  // (tile, k-block)
        const int64_t tile = block / k_blocks, kb = block % k_blocks;
        const int64_t row = pair_offset > 0 ? (r < 64 ? tile * 64 + r : pair_offset + tile * 64 + (r - 64))
                                            : tile * 128 + r;
        const int lc = pc ^ (r & 7);
        reinterpret_cast<uint4*>(packed)[q] =
            *reinterpret_cast<const uint4*>(w + row * in_features + kb * 64 + lc * 8);
    }
}

// ------------------------------------------------------------------ host side
struct ProjPlan {
    int nt, chunks, split, stages, tmem_cols, smem;
};

// Largest cluster the device schedules for this kernel at this shared-memory
// size: 16 (non-portable, opted in here) when it fits, else the portable 8.
static int proj_cluster_limit(void (*kernel)(ProjParams), int smem) {
    int best = 8;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(kProjMaxSplit, 1, 1);
        cfg.blockDim = dim3(kProjThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = kProjMaxSplit;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess && clusters > 0)
            best = kProjMaxSplit;
    }
    cudaGetLastError();
    return best;
}

static int next_pow2_at_least(int x, int lo) {
    int v = lo;
    while (v < x) v <<= 1;
    return v;
}

// Tokens per CTA (NT, the UMMA N): a multiple of 16, at most kProjMaxTokens.
static int proj_tile_tokens(int64_t tokens) {
    return (int)std::min<int64_t>(kProjMaxTokens, (std::max<int64_t>(tokens, 1) + 15) / 16 * 16);
}

// Tokens per CTA, split-K and ring depth for `tiles` output tiles (graph-static).
static ProjPlan make_proj_plan(int64_t tokens, int64_t in_features, int64_t tiles, int sm_count, int max_split) {
    ProjPlan pl{};
    pl.nt = proj_tile_tokens(tokens);
    pl.chunks = (int)((tokens + pl.nt - 1) / pl.nt);
    const int kb = (int)(in_features / 64);
    const int64_t base = tiles * pl.chunks;
    // small batches fit two CTAs per SM: aim at two per SM, else one
    const int64_t target = (int64_t)sm_count * (pl.nt <= 64 ? 2 : 1);
    const int64_t want = std::max<int64_t>(1, std::min<int64_t>({target / std::max<int64_t>(1, base),
                                                                 (int64_t)kb, (int64_t)max_split}));
    pl.split = 1;  // a power of two, so that clusters tile the GPCs evenly
    while (pl.split * 2 <= want) pl.split *= 2;
    const int stage = kProjWBytes + pl.nt * 128;
    const int max_kb = (kb + pl.split - 1) / pl.split;
    // small batches: two CTAs per SM, so that the next chained projection's CTAs fit beside
    const int budget = pl.nt <= 64 ? 112 * 1024 : 200 * 1024;
    const int fixed = ProjLayout(pl.nt, 0, pl.split).smem - pl.nt * 512;  // everything but the ring
    pl.stages = std::max(1, std::min({kProjMaxStages, max_kb, (budget - fixed) / stage}));
    pl.tmem_cols = next_pow2_at_least(pl.nt, 32);
    pl.smem = ProjLayout(pl.nt, pl.stages, pl.split).smem;
    return pl;
}

template <typename T, int EPI, bool NORM>
static cudaError_t launch_proj_typed(ProjParams p, int64_t tiles, cudaStream_t stream) {
    auto kernel = proj_kernel<T, EPI, NORM>;
    static int configured[64] = {0};  // the attribute is per device: set on each device the kernel runs on
    cudaError_t set = ensure_smem_limit(kernel, 232448 - 1024, configured);
    if (set != cudaSuccess) return set;
    // cluster limit of this kernel, cached per device and shared-memory size
    struct ClusterLimit {
        int smem = -1, limit = 8;
    };
    static ClusterLimit limits[64];
    int limit = 8;
    const ProjPlan probe = make_proj_plan(p.tokens, p.in_features, tiles, sm_count(), kProjMaxSplit);
    if (probe.split > 8) {
        int device = 0;
        if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) device = -1;
        std::lock_guard<std::mutex> guard(g_smem_attribute_lock);
        if (device < 0) {
            limit = proj_cluster_limit(kernel, probe.smem);
        } else {
            ClusterLimit& cached = limits[device];
            if (cached.smem != probe.smem) cached = ClusterLimit{probe.smem, proj_cluster_limit(kernel, probe.smem)};
            limit = cached.limit;
        }
    }
    const ProjPlan pl = probe.split > 8 && limit < probe.split
                            ? make_proj_plan(p.tokens, p.in_features, tiles, sm_count(), limit)
                            : probe;
    p.tile_tokens = pl.nt;
    p.split = pl.split;
    p.stages = pl.stages;
    p.tmem_cols = pl.tmem_cols;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)pl.split, (unsigned)tiles, (unsigned)pl.chunks);
    cfg.blockDim = dim3(kProjThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)pl.split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, p);
}

template <int EPI>
static cudaError_t launch_proj(int dtype, bool norm, const ProjParams& p, int64_t tiles, cudaStream_t s) {
    if (dtype == MINIKV_BF16)
        return norm ? launch_proj_typed<__nv_bfloat16, EPI, true>(p, tiles, s)
                    : launch_proj_typed<__nv_bfloat16, EPI, false>(p, tiles, s);
    return norm ? launch_proj_typed<__half, EPI, true>(p, tiles, s)
                : launch_proj_typed<__half, EPI, false>(p, tiles, s);
}

// Shared checks of every projection entry point (`weight_rows` rows of the
// packed weight).
static int proj_setup(const void* x, int64_t x_stride, const void* packed_weight, int64_t tokens,
                      int64_t in_features, int64_t weight_rows, const float* ss_in, const void* norm_weight, int dtype,
                      ProjParams* p) {
    if (dtype != MINIKV_BF16 && dtype != MINIKV_F16) return fail(MINIKV_EINVAL, "projections run in fp16 or bf16");
    if (tokens < 0 || tokens >= (1ll << 31) || in_features <= 0 || in_features % 64 != 0 ||
        in_features >= (1ll << 31) || weight_rows <= 0 || weight_rows >= (1ll << 31))
        return fail(MINIKV_EINVAL, "projection sizes: in_features must be a positive multiple of 64");
    if (x_stride < in_features || (x_stride * 2) % 16 != 0)
        return fail(MINIKV_EINVAL, "projection input rows must be 16-byte aligned and hold in_features");
    if (x == nullptr || packed_weight == nullptr || !aligned16(x) || !aligned16(packed_weight))
        return fail(MINIKV_EINVAL, "projection operands must be 16-byte aligned");
    if (ss_in != nullptr && (norm_weight == nullptr || in_features % 128 != 0))
        return fail(MINIKV_EINVAL, "the RMSNorm prologue needs its weight and in_features % 128 == 0");
    *p = ProjParams{};
    p->w = packed_weight;
    p->x = x;
    p->x_stride = x_stride;
    p->tokens = (int)tokens;
    p->in_features = (int)in_features;
    p->k_blocks = (int)(in_features / 64);
    p->ss_in = ss_in;
    p->norm_weight = norm_weight;
    return MINIKV_OK;
}

static cudaError_t launch_pack_linear(int dtype, const void* w, void* packed, int64_t rows, int64_t in_features,
                                      int64_t pair_offset, int sms, cudaStream_t s) {
    const int64_t chunks = rows * in_features / 8;
    const int64_t blocks = std::min<int64_t>((chunks + 255) / 256, (int64_t)sms * 8);
    const int kb = (int)(in_features / 64);
    if (dtype == MINIKV_BF16)
        pack_linear_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(w), static_cast<__nv_bfloat16*>(packed), chunks, kb, in_features,
            pair_offset);
    else
        pack_linear_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(static_cast<const __half*>(w),
                                                                   static_cast<__half*>(packed), chunks, kb,
                                                                   in_features, pair_offset);
    return cudaGetLastError();
}

}  // namespace minikv
