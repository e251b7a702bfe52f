// KV writes: packed scatter by slot, decode append, contiguous range, and
// copy-on-write of whole pages.  Pure byte moves: one warp per token row,
// 16-byte vector loads/stores, grid sized to the SM count (grid-stride).
// Launched as chained kernels: each waits for the previous kernel first and
// then lets the next one (typically the decode of the same step) launch.
//
// Reference behaviour kept (mini_engine/kernels/csrc/data.cu):
//  * rows whose destination is out of range are skipped, never clamped
//    (data.cu:77-79, :98-100, :200-201);
//  * results are bit-exact copies of the source rows.
#include "common.cuh"

namespace minikv {

// Row destination for the three write forms.  Returns -1 for "skip".
struct SlotRows {         // data.cu:196-206
    const int64_t* slots;
    int64_t capacity;
    __device__ int64_t operator()(int64_t t) const {
        const int64_t s = slots[t];
        return (s >= 0 && s < capacity) ? s : -1;
    }
};
struct AppendRows {       // data.cu:89-107
    const int64_t* tables; const int64_t* offsets;
    int64_t width, num_blocks, block_size;
    __device__ int64_t operator()(int64_t r) const {
        const int64_t logical = offsets[r];
        if (logical < 0) return -1;
        const int64_t index = logical / block_size;
        if (index >= width) return -1;
        const int64_t page = tables[r * width + index];
        if (page < 0 || page >= num_blocks) return -1;
        return page * block_size + logical % block_size;
    }
};
struct RangeRows {        // data.cu:68-86
    const int64_t* ids; int64_t num_ids, offset, num_blocks, block_size;
    __device__ int64_t operator()(int64_t t) const {
        const int64_t logical = offset + t;
        const int64_t index = logical / block_size;
        if (logical < 0 || index >= num_ids) return -1;
        const int64_t page = ids[index];
        if (page < 0 || page >= num_blocks) return -1;
        return page * block_size + logical % block_size;
    }
};

// One warp copies the K row and the V row of one token; rows are
// `row_vecs` 16-byte vectors long.
template <typename Rows>
__global__ void __launch_bounds__(256) write_rows_kernel(
    uint4* __restrict__ kc, uint4* __restrict__ vc, const uint4* __restrict__ k,
    const uint4* __restrict__ v, int64_t rows, int64_t row_vecs, int64_t k_stride_vecs,
    int64_t v_stride_vecs, Rows map) {
    griddep_wait();
    griddep_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < rows; t += warps) {
        const int64_t dst = map(t);
        if (dst < 0) continue;
        const uint4* ks = k + t * k_stride_vecs;
        const uint4* vs = v + t * v_stride_vecs;
        uint4* kd = kc + dst * row_vecs;
        uint4* vd = vc + dst * row_vecs;
        for (int64_t c = lane; c < row_vecs; c += 32) {
            const uint4 a = ld_global_nc(ks + c);
            const uint4 b = ld_global_nc(vs + c);
            kd[c] = a;
            vd[c] = b;
        }
    }
}

// Copy-on-write: unit u = (pair, layer, K|V) copies one page of
// `page_vecs` 16-byte vectors.  One CTA per unit, grid-stride over units.
__global__ void __launch_bounds__(256) copy_blocks_kernel(
    uint4* __restrict__ kpool, uint4* __restrict__ vpool, const int64_t* __restrict__ pairs,
    int64_t num_pairs, int64_t num_layers, int64_t num_blocks, int64_t page_vecs) {
    griddep_wait();
    griddep_launch_dependents();
    const int64_t units = num_pairs * num_layers * 2;
    for (int64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const int64_t pair = u / (num_layers * 2);
        const int64_t layer = (u / 2) % num_layers;
        uint4* pool = (u & 1) ? vpool : kpool;
        const int64_t src = pairs[2 * pair], dst = pairs[2 * pair + 1];
        if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) continue;
        const uint4* s = pool + (layer * num_blocks + src) * page_vecs;
        uint4* d = pool + (layer * num_blocks + dst) * page_vecs;
        for (int64_t c = threadIdx.x; c < page_vecs; c += blockDim.x) d[c] = ld_global_nc(s + c);
    }
}

static int sm_count_for_current_device() {
    static int cached[64] = {0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
    if (cached[device] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        cached[device] = n > 0 ? n : 148;
    }
    return cached[device];
}

template <typename Rows>
static cudaError_t launch_write_rows(void* kc, void* vc, const void* k, const void* v, int64_t rows,
                                     int64_t row_bytes, int64_t k_stride_bytes, int64_t v_stride_bytes,
                                     Rows map, cudaStream_t stream) {
    if (rows <= 0) return cudaSuccess;
    const int64_t per_block = 8;  // warps
    int64_t blocks = (rows + per_block - 1) / per_block;
    const int64_t cap = (int64_t)sm_count_for_current_device() * 8;
    if (blocks > cap) blocks = cap;
    return launch_chained(write_rows_kernel<Rows>, dim3((unsigned)blocks), dim3(256), 0, stream,
                          static_cast<uint4*>(kc), static_cast<uint4*>(vc), static_cast<const uint4*>(k),
                          static_cast<const uint4*>(v), rows, row_bytes / 16, k_stride_bytes / 16,
                          v_stride_bytes / 16, map);
}

static cudaError_t launch_copy_blocks(void* kpool, void* vpool, const int64_t* pairs, int64_t num_pairs,
                                      int64_t num_layers, int64_t num_blocks, int64_t page_bytes,
                                      cudaStream_t stream) {
    const int64_t units = num_pairs * num_layers * 2;
    if (units <= 0) return cudaSuccess;
    int64_t blocks = units;
    const int64_t cap = (int64_t)sm_count_for_current_device() * 8;
    if (blocks > cap) blocks = cap;
    return launch_chained(copy_blocks_kernel, dim3((unsigned)blocks), dim3(256), 0, stream,
                          static_cast<uint4*>(kpool), static_cast<uint4*>(vpool), pairs, num_pairs, num_layers,
                          num_blocks, page_bytes / 16);
}

}  // namespace minikv
