// assemble.cu -- split-N output assembly after an all-gather.
//
// Column-parallel sharding gives rank r the output columns [r*ns, (r+1)*ns).  An all-gather
// of the per-rank [rows][ns] slabs leaves them back to back ([shards][rows][ns]); the
// consumer wants [rows][shards*ns].  One pass, 16-byte loads and stores when the slab
// width allows (HBM-bound: every byte read once and written once).
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace ql {

namespace {

template <typename V>
__global__ void interleave_kernel(const V *__restrict__ src, V *__restrict__ dst, int shards,
                                  int rows, int vec_per_row) {
    const long long per_shard = (long long)rows * vec_per_row;
    const long long total = per_shard * shards;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int s = (int)(i / per_shard);
        const long long r = i % per_shard;
        const long long m = r / vec_per_row;
        const int j = (int)(r % vec_per_row);
        dst[(m * shards + s) * vec_per_row + j] = src[i];
    }
}

}  // namespace

cudaError_t launch_interleave(const void *src, void *dst, int shards, int rows, int shard_cols,
                              int elem_bytes, int num_sms, cudaStream_t stream) {
    const long long row_bytes = (long long)shard_cols * elem_bytes;
    const long long total_bytes = row_bytes * rows * shards;
    int grid = (int)std::min<long long>((total_bytes / 16 + 255) / 256, (long long)num_sms * 8);
    if (grid < 1) grid = 1;
    const bool v16 = row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(dst) & 15) == 0;
    if (v16)
        interleave_kernel<uint4><<<grid, 256, 0, stream>>>(
            static_cast<const uint4 *>(src), static_cast<uint4 *>(dst), shards, rows,
            (int)(row_bytes / 16));
    else if (elem_bytes == 4)
        interleave_kernel<uint32_t><<<grid, 256, 0, stream>>>(
            static_cast<const uint32_t *>(src), static_cast<uint32_t *>(dst), shards, rows,
            shard_cols);
    else if (elem_bytes == 2)
        interleave_kernel<uint16_t><<<grid, 256, 0, stream>>>(
            static_cast<const uint16_t *>(src), static_cast<uint16_t *>(dst), shards, rows,
            shard_cols);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace ql
