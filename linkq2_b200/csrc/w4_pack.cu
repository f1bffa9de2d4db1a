// Load-time int4 packing: values [N, K] int8 -> packed [K/8, N] int32.
// Replaces pack_weights_over_cols_triton(codes, 4, 32, transpose=True).contiguous()
// (qslab/kernels/gemlite/bitpack.py:63-125) and the +8 offset of symmetric
// checkpoints (qslab/runtime/backends/gemlite.py:22-23).  Bit-exact by construction:
// word(k8, n) = OR_j ((values[n, 8*k8 + j] + offset) & 15) << 4j.
#include "common.cuh"

namespace lq2 {

namespace {

// 32 output columns (n) x 32 words (k8) per CTA, transposed through shared
// memory so that both the byte reads (along K) and the word writes (along N)
// are coalesced.
__global__ void __launch_bounds__(256) w4_pack_kernel(const int8_t* __restrict__ values, int offset,
                                                      int32_t* __restrict__ packed, int n, int k8_total) {
    __shared__ uint32_t tile[32][33];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    const int nb = blockIdx.x * 32, kb = blockIdx.y * 32;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int nn = nb + ty + 8 * r, k8 = kb + tx;
        uint32_t word = 0;
        if (nn < n && k8 < k8_total) {
            const uint2 raw = *reinterpret_cast<const uint2*>(values + (int64_t(nn) * k8_total + k8) * 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t byte = ((j < 4 ? raw.x : raw.y) >> (8 * (j & 3))) & 0xff;
                word |= ((byte + uint32_t(offset)) & 15u) << (4 * j);
            }
        }
        tile[ty + 8 * r][tx] = word;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int k8 = kb + ty + 8 * r, nn = nb + tx;
        if (nn < n && k8 < k8_total) packed[int64_t(k8) * n + nn] = int32_t(tile[tx][ty + 8 * r]);
    }
}

}  // namespace

int w4_pack_launch(const int8_t* values, int offset, int32_t* packed, int n, int k, cudaStream_t st) {
    dim3 grid(cdiv(n, 32), cdiv(k / 8, 32));
    w4_pack_kernel<<<grid, 256, 0, st>>>(values, offset, packed, n, k / 8);
    return check_launch();
}

}  // namespace lq2
