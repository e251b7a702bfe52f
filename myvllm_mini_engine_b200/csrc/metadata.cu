// Device-side metadata construction.
//
// prefill: the seven tensors of PrefillBatch.from_sequences
//   (mini_engine/engine/batch.py:67-137) from compact per-request inputs, so the
//   host loops over requests and pages only, never over tokens.
// decode:  the fixed-shape tables of a CUDA-graph bucket
//   (mini_engine/engine/cuda_graph.py:149-181, padding rows :66-86) from the
//   active requests' block lists; the active count is read on the device.
// Also the token -> (request, context length) map used by the CUDA-core
// prefill route (prefill.cu:112-123 computes the same per-token quantities).
#include "common.cuh"

namespace minikv {

__global__ void __launch_bounds__(256) prefill_metadata_kernel(
    const int64_t* __restrict__ starts, const int64_t* __restrict__ cu_q, const int64_t* __restrict__ cu_blocks,
    const int64_t* __restrict__ block_ids, const int64_t* __restrict__ token_ids, int64_t requests,
    int64_t width, int64_t block_size, int64_t* __restrict__ input_ids, int64_t* __restrict__ positions,
    int64_t* __restrict__ slots, int64_t* __restrict__ out_cu, int64_t* __restrict__ out_starts,
    int64_t* __restrict__ context_lens, int64_t* __restrict__ tables) {
    for (int64_t r = blockIdx.x; r < requests; r += gridDim.x) {
        const int64_t start = starts[r], q0 = cu_q[r], q1 = cu_q[r + 1];
        const int64_t b0 = cu_blocks[r], nb = cu_blocks[r + 1] - b0;
        for (int64_t i = q0 + threadIdx.x; i < q1; i += blockDim.x) {
            const int64_t pos = start + (i - q0);                 // batch.py:110-118
            const int64_t index = pos / block_size;
            const int64_t page = (pos >= 0 && index < nb) ? block_ids[b0 + index] : -1;
            input_ids[i] = token_ids[i];
            positions[i] = pos;
            slots[i] = page >= 0 ? page * block_size + pos % block_size : -1;
        }
        for (int64_t j = threadIdx.x; j < width; j += blockDim.x)   // batch.py:128-129
            tables[r * width + j] = j < nb ? block_ids[b0 + j] : -1;
        if (threadIdx.x == 0) {
            out_cu[r] = q0;
            if (r == requests - 1) out_cu[requests] = q1;
            out_starts[r] = start;
            context_lens[r] = start + (q1 - q0);
        }
    }
}

__global__ void __launch_bounds__(128) decode_tables_kernel(
    const int64_t* __restrict__ active, const int64_t* __restrict__ tokens, const int64_t* __restrict__ positions,
    const int64_t* __restrict__ cu_blocks, const int64_t* __restrict__ block_ids,
    const int64_t* __restrict__ padding, int64_t batch, int64_t width, int64_t* __restrict__ out_ids,
    int64_t* __restrict__ out_positions, int64_t* __restrict__ tables) {
    const int64_t count = *active;
    for (int64_t r = blockIdx.x; r < batch; r += gridDim.x) {
        if (r < count) {
            const int64_t b0 = cu_blocks[r], nb = cu_blocks[r + 1] - b0;
            for (int64_t j = threadIdx.x; j < width; j += blockDim.x)
                tables[r * width + j] = j < nb ? block_ids[b0 + j] : -1;
            if (threadIdx.x == 0) {
                out_ids[r] = tokens[r];
                out_positions[r] = positions[r];
            }
        } else {  // padding row: position 0 on its private scratch page
            for (int64_t j = threadIdx.x; j < width; j += blockDim.x)
                tables[r * width + j] = j == 0 ? padding[r] : -1;
            if (threadIdx.x == 0) {
                out_ids[r] = 0;
                out_positions[r] = 0;
            }
        }
    }
}

// Packed query token t -> (request row, context length t attends).  Tokens of
// malformed metadata get length 0, which the decode kernel turns into zeros.
__global__ void __launch_bounds__(256) prefill_token_map_kernel(
    const int64_t* __restrict__ cu_q, const int64_t* __restrict__ starts, const int64_t* __restrict__ lens,
    int64_t requests, int64_t first_token, int64_t tokens, int64_t width, int64_t block_size,
    int64_t* __restrict__ token_len, int64_t* __restrict__ token_row) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < tokens;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = first_token + i;
        int64_t lo = 0, hi = requests;  // first r with cu_q[r + 1] > t
        while (lo < hi) {
            const int64_t mid = (lo + hi) / 2;
            if (cu_q[mid + 1] <= t) lo = mid + 1; else hi = mid;
        }
        int64_t len = 0, row = 0;
        if (lo < requests && t >= cu_q[lo]) {
            const int64_t last = starts[lo] + t - cu_q[lo];
            if (last >= 0 && last < lens[lo] && last / block_size < width) len = last + 1;
            row = lo;
        }
        token_len[i] = len;
        token_row[i] = row;
    }
}

}  // namespace minikv
