// W4A16 linear for small M (decode GEMV, batched decode, 16-position verify):
// a weight-streaming kernel bounded by HBM bandwidth.
//
// Replaces the GEMV and split-K Triton routes of the reference
// (qslab/kernels/gemlite/triton_kernels/gemv_revsplitK_A16fWnO16f_int32packing.py:155-384,
//  gemm_splitK_A16fWnO16f_int32packing.py:199-412) behind the same buffers:
//   packed [K/8, N] int32 (n fastest; nibble j of word (k8, n) is k = 8*k8 + j),
//   scales / zeros [K/group, N] fp16.
//
// Data movement.  A CTA of WN warps owns 32*WN output columns and a contiguous
// range of K.  Packed words, scales, zero points and activations are copied
// global -> shared with cp.async through a ring of STAGES buffers of 128 k each,
// so the bytes in flight per SM are set by the ring depth, not by registers.
// Lane (g, t) = (lane / 4, lane % 4) of a warp then reads one 128-bit word quad
// per 32-k step, packed[k8 = 4*step + t][n0 .. n0+3] with n0 = 32*warp + 4*g; the
// row pitch of the ring is padded by 32 bytes so these reads are conflict-free.
// Nibbles are unpacked in registers and fed to the warp-level tensor-core op
// m16n8k16 used as a dot-product engine: the MMA's 16 "rows" are output columns
// (two per lane group), its 16 k-slots are the eight nibbles of lane t's words
// in an order chosen so that unpacking needs one shift per word (the activation
// fragment is permuted to match with four byte-permutes), and its 8 "columns"
// are activation rows.  The four lanes of a group hold different k, so the MMA
// performs the cross-lane reduction itself.
//
// For M <= 8 the group scale is applied after the group's integer dot product:
//   y += s * (sum_k (u - 8) x_k  -  (z - 8) * sum_k x_k)
// with the activation sum produced by one extra MMA against a fragment of ones.
// For 8 < M <= 64 weights are dequantised to fp16 exactly as the reference does,
// (u - z) * s rounded once (triton_kernels/utils.py:66-71; zero points must be
// integer valued, which every reference quantizer guarantees), and accumulated
// in fp32.
//
// Split-K.  The CTAs that share a column tile form a thread-block cluster along
// grid.y.  Each leaves its fp32 partial tile in its own shared memory; after a
// cluster barrier every CTA sums one slice of the columns over all ranks through
// distributed shared memory, in rank order (so the result does not depend on
// timing), and writes fp16.  No global scratch, no atomics.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lq2 {

namespace {

constexpr int kStageK = 128;                     // k per pipeline stage
constexpr int kXsRowBytes = kStageK * 2 + 64;    // +64: conflict-free 128-bit fragment loads

struct W4Params {
    const __half* x;
    int64_t ldx;
    const int32_t* packed;
    const __half* scales;
    const __half* zeros;
    __half* y;
    int m, n, k, group;
    int stages_per_rank;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const int bytes = pred ? 16 : 0;             // 0 source bytes: the 16 destination bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ uint32_t bcast_half(uint2 v, int idx) {
    const uint32_t w = idx < 2 ? v.x : v.y;
    return __byte_perm(w, w, (idx & 1) ? 0x3232 : 0x1010);
}
__device__ __forceinline__ float half_at(uint2 v, int idx) {
    const uint32_t w = idx < 2 ? v.x : v.y;
    return __half2float(__ushort_as_half((unsigned short)((idx & 1) ? (w >> 16) : (w & 0xffff))));
}

template <int NJ, int WN, int GPS>
struct Layout {
    static constexpr int MT = 8 * NJ;
    static constexpr int TN = 32 * WN;
    static constexpr int WROW = TN * 4 + 32;                 // bytes per packed row in the ring
    static constexpr int W_BYTES = 16 * WROW;
    static constexpr int X_BYTES = MT * kXsRowBytes;
    static constexpr int S_BYTES = GPS * TN * 2;
    static constexpr int STAGE_BYTES = W_BYTES + X_BYTES + 2 * S_BYTES;
    static constexpr int STAGES = NJ == 1 ? 6 : (NJ == 2 ? 6 : (NJ == 4 ? 5 : 4));
    static constexpr int RED_BYTES = MT * TN * 4;
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr int SMEM_BYTES = RING_BYTES > RED_BYTES ? RING_BYTES : RED_BYTES;
};

template <int NJ, bool ZTABLE, int GPS, int WN>
__global__ void __launch_bounds__(32 * WN, (NJ <= 2 ? 4 : 2)) w4a16_stream_kernel(const W4Params p) {
    using L = Layout<NJ, WN, GPS>;
    constexpr bool SCALE_AFTER = (NJ == 1);
    constexpr int MT = L::MT, TN = L::TN, THREADS = 32 * WN, STAGES = L::STAGES;
    constexpr int STEPS_PER_GROUP = 4 / GPS;

    extern __shared__ __align__(128) unsigned char smem[];

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int m0 = blockIdx.z * MT;
    const int rows = min(MT, p.m - m0);
    const int tile_n0 = blockIdx.x * TN;
    const int nb = tile_n0 + warp * 32;
    const bool n_ok = nb < p.n;
    const int n0 = nb + 4 * g;
    const int k8_total = p.k >> 3;
    const int total_stages = (p.k + kStageK - 1) / kStageK;
    const int ranks = gridDim.y, rank = blockIdx.y;
    const int s0 = min(total_stages, rank * p.stages_per_rank);
    const int s1 = min(total_stages, s0 + p.stages_per_rank);
    const int my_stages = s1 - s0;
    const int groups_total = p.k / p.group;

    auto issue = [&](int s, int buf) {
        unsigned char* base = smem + buf * L::STAGE_BYTES;
        // packed words: 16 rows x TN columns, 16-byte chunks
        constexpr int WCHUNKS = 16 * (TN / 4);
#pragma unroll
        for (int c = tid; c < WCHUNKS; c += THREADS) {
            const int row = c / (TN / 4), col4 = c % (TN / 4);
            const int k8 = s * 16 + row, nn = tile_n0 + col4 * 4;
            const bool ok = k8 < k8_total && nn < p.n;
            cp_async16(base + row * L::WROW + col4 * 16, ok ? (const void*)(p.packed + int64_t(k8) * p.n + nn) : (const void*)p.packed, ok);
        }
        // activations: MT rows x 128 k, raw order
        unsigned char* xb = base + L::W_BYTES;
        constexpr int XCHUNKS = MT * 16;
#pragma unroll
        for (int c = tid; c < XCHUNKS; c += THREADS) {
            const int row = c >> 4, kc = c & 15;
            const int kk = s * kStageK + kc * 8;
            const bool ok = row < rows && kk < p.k;
            cp_async16(xb + row * kXsRowBytes + kc * 16, ok ? (const void*)(p.x + int64_t(m0 + row) * p.ldx + kk) : (const void*)p.x, ok);
        }
        // scales / zero points of the stage's groups: GPS rows x TN halves
        unsigned char* sb = xb + L::X_BYTES;
        constexpr int SCHUNKS = GPS * (TN / 8);
        for (int c = tid; c < SCHUNKS; c += THREADS) {
            const int q = c / (TN / 8), col8 = c % (TN / 8);
            int gi = (GPS == 1) ? (s * kStageK) / p.group : s * GPS + q;
            gi = min(gi, groups_total - 1);
            const int nn = tile_n0 + col8 * 8;
            const bool ok = nn < p.n;
            cp_async16(sb + q * TN * 2 + col8 * 16, ok ? (const void*)(p.scales + int64_t(gi) * p.n + nn) : (const void*)p.scales, ok);
            if (ZTABLE)
                cp_async16(sb + L::S_BYTES + q * TN * 2 + col8 * 16, ok ? (const void*)(p.zeros + int64_t(gi) * p.n + nn) : (const void*)p.scales, ok);
        }
    };

    float acc[2][NJ][4];
    float gacc[2][SCALE_AFTER ? NJ : 1][4];
    float xsum[SCALE_AFTER ? NJ : 1][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) gacc[i][0][c] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) xsum[0][c] = 0.f;

    const __half2 k1032 = __floats2half2_rn(1032.f, 1032.f);
    const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
    const __half2 km72 = __floats2half2_rn(-72.f, -72.f);
    const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
    const __half2 k64 = __floats2half2_rn(64.f, 64.f);
    constexpr uint32_t kOnes = 0x3C003C00u;

#pragma unroll
    for (int i = 0; i < STAGES - 1; ++i) {
        if (i < my_stages) issue(s0 + i, i);
        cp_async_commit();
    }

    for (int it = 0; it < my_stages; ++it) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            const int nxt = it + STAGES - 1;
            if (nxt < my_stages) issue(s0 + nxt, nxt % STAGES);
            cp_async_commit();
        }
        const unsigned char* base = smem + (it % STAGES) * L::STAGE_BYTES;
        const unsigned char* wsm = base + warp * 128 + g * 16;
        const unsigned char* xsm = base + L::W_BYTES;
        const unsigned char* ssm = xsm + L::X_BYTES + warp * 64 + g * 8;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint4 wq = *reinterpret_cast<const uint4*>(wsm + (kk * 4 + t) * L::WROW);
            const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
            uint4 xb[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const uint4 r = *reinterpret_cast<const uint4*>(xsm + (8 * j + g) * kXsRowBytes + (kk * 4 + t) * 16);
                // halves x0..x7 -> {x0,x4} {x1,x5} {x2,x6} {x3,x7}: the k-slot order of the A fragments
                xb[j].x = __byte_perm(r.x, r.z, 0x5410);
                xb[j].y = __byte_perm(r.x, r.z, 0x7632);
                xb[j].z = __byte_perm(r.y, r.w, 0x5410);
                xb[j].w = __byte_perm(r.y, r.w, 0x7632);
            }
            const int gq = kk / STEPS_PER_GROUP;
            uint2 sc = make_uint2(0, 0), zc = make_uint2(0, 0);
            if (!SCALE_AFTER || (kk + 1) % STEPS_PER_GROUP == 0) {
                sc = *reinterpret_cast<const uint2*>(ssm + gq * TN * 2);
                if (ZTABLE) zc = *reinterpret_cast<const uint2*>(ssm + L::S_BYTES + gq * TN * 2);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                __half2 s_a, s_b, zlo_a, zlo_b, zhi_a, zhi_b;
                if (!SCALE_AFTER) {
                    s_a = u32_as_h2(bcast_half(sc, 2 * i));
                    s_b = u32_as_h2(bcast_half(sc, 2 * i + 1));
                    if (ZTABLE) {
                        const __half2 z_a = u32_as_h2(bcast_half(zc, 2 * i));
                        const __half2 z_b = u32_as_h2(bcast_half(zc, 2 * i + 1));
                        zlo_a = __hadd2(z_a, k1024);
                        zlo_b = __hadd2(z_b, k1024);
                        zhi_a = __hneg2(__hadd2(z_a, k64));
                        zhi_b = __hneg2(__hadd2(z_b, k64));
                    } else {
                        zlo_a = zlo_b = k1032;
                        zhi_a = zhi_b = km72;
                    }
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t wa = wv[2 * i] >> (8 * h);
                    const uint32_t wb = wv[2 * i + 1] >> (8 * h);
                    const __half2 lo_a = u32_as_h2(and_or(wa, 0x000f000fu, 0x64006400u));
                    const __half2 hi_a = u32_as_h2(and_or(wa, 0x00f000f0u, 0x64006400u));
                    const __half2 lo_b = u32_as_h2(and_or(wb, 0x000f000fu, 0x64006400u));
                    const __half2 hi_b = u32_as_h2(and_or(wb, 0x00f000f0u, 0x64006400u));
                    uint32_t a0, a1, a2, a3;
                    if (SCALE_AFTER) {
                        a0 = h2_as_u32(__hsub2(lo_a, k1032));
                        a1 = h2_as_u32(__hsub2(lo_b, k1032));
                        a2 = h2_as_u32(__hfma2(hi_a, k16th, km72));
                        a3 = h2_as_u32(__hfma2(hi_b, k16th, km72));
                    } else {
                        a0 = h2_as_u32(__hmul2(__hsub2(lo_a, zlo_a), s_a));
                        a1 = h2_as_u32(__hmul2(__hsub2(lo_b, zlo_b), s_b));
                        a2 = h2_as_u32(__hmul2(__hfma2(hi_a, k16th, zhi_a), s_a));
                        a3 = h2_as_u32(__hmul2(__hfma2(hi_b, k16th, zhi_b), s_b));
                    }
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        const uint32_t b0 = h ? xb[j].z : xb[j].x;
                        const uint32_t b1 = h ? xb[j].w : xb[j].y;
                        if constexpr (SCALE_AFTER) mma_m16n8k16(gacc[i][j], a0, a1, a2, a3, b0, b1);
                        else mma_m16n8k16(acc[i][j], a0, a1, a2, a3, b0, b1);
                    }
                }
            }
            if constexpr (SCALE_AFTER) {
                if (ZTABLE) {
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        mma_m16n8k16(xsum[j], kOnes, kOnes, kOnes, kOnes, xb[j].x, xb[j].y);
                        mma_m16n8k16(xsum[j], kOnes, kOnes, kOnes, kOnes, xb[j].z, xb[j].w);
                    }
                }
                if ((kk + 1) % STEPS_PER_GROUP == 0) {
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        const float sa = half_at(sc, 2 * i), sb = half_at(sc, 2 * i + 1);
                        float za = 0.f, zb = 0.f;
                        if (ZTABLE) {
                            za = half_at(zc, 2 * i) - 8.f;
                            zb = half_at(zc, 2 * i + 1) - 8.f;
                        }
#pragma unroll
                        for (int j = 0; j < NJ; ++j) {
                            acc[i][j][0] += sa * (gacc[i][j][0] - za * xsum[j][0]);
                            acc[i][j][1] += sa * (gacc[i][j][1] - za * xsum[j][1]);
                            acc[i][j][2] += sb * (gacc[i][j][2] - zb * xsum[j][0]);
                            acc[i][j][3] += sb * (gacc[i][j][3] - zb * xsum[j][1]);
#pragma unroll
                            for (int c = 0; c < 4; ++c) gacc[i][j][c] = 0.f;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < NJ; ++j)
#pragma unroll
                        for (int c = 0; c < 4; ++c) xsum[j][c] = 0.f;
                }
            }
        }
    }
    cp_async_wait<0>();

    // ---- write-out.  Lane (g, t) owns columns n0..n0+3 of rows m0 + 8j + 2t (+1).
    if (ranks == 1) {
        if (n_ok) {
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const int m = m0 + 8 * j + 2 * t + r;
                    if (m < p.m) {
                        const __half2 lo = __floats2half2_rn(acc[0][j][r], acc[0][j][2 + r]);
                        const __half2 hi = __floats2half2_rn(acc[1][j][r], acc[1][j][2 + r]);
                        *reinterpret_cast<uint2*>(p.y + int64_t(m) * p.n + n0) =
                            make_uint2(h2_as_u32(lo), h2_as_u32(hi));
                    }
                }
            }
        }
        return;
    }

    // ---- cluster reduction through distributed shared memory
    cg::cluster_group cluster = cg::this_cluster();
    __syncthreads();                                   // every warp is done with the ring
    float* red = reinterpret_cast<float*>(smem);       // [MT][TN]
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int ml = 8 * j + 2 * t + r;
            *reinterpret_cast<float4*>(red + ml * TN + warp * 32 + 4 * g) =
                make_float4(acc[0][j][r], acc[0][j][2 + r], acc[1][j][r], acc[1][j][2 + r]);
        }
    }
    cluster.sync();
    {
        const int slice = TN / ranks;                  // columns this rank finishes (ranks <= 8 divides TN)
        const int c0 = rank * slice;
        const int quads = slice / 4;
        for (int e = tid; e < rows * quads; e += THREADS) {
            const int ml = e / quads, cq = e % quads;
            const int col = c0 + cq * 4;
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < ranks; ++q) {
                const float* remote = cluster.map_shared_rank(red, q);
                const float4 v = *reinterpret_cast<const float4*>(remote + ml * TN + col);
                sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
            }
            const int nn = tile_n0 + col;
            if (nn < p.n) {
                const __half2 lo = __floats2half2_rn(sum.x, sum.y);
                const __half2 hi = __floats2half2_rn(sum.z, sum.w);
                *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * p.n + nn) = make_uint2(h2_as_u32(lo), h2_as_u32(hi));
            }
        }
    }
    cluster.sync();                                    // nobody leaves while its tile is still being read
}

struct Plan {
    int nj, wn, m_tiles, n_tiles, ranks, spr;
};

Plan make_plan(int m, int n, int k) {
    Plan p;
    p.nj = m <= 8 ? 1 : (m <= 16 ? 2 : (m <= 32 ? 4 : 8));
    p.m_tiles = cdiv(m, 8 * p.nj);
    const int stages = cdiv(k, kStageK);
    const int target = 2 * kNumSMs;
    // 128-column tiles when that alone (times the largest cluster) fills the machine, else 64
    p.wn = (cdiv(n, 128) * p.m_tiles * 8 >= target) ? 4 : 2;
    p.n_tiles = cdiv(n, 32 * p.wn);
    const int base = p.n_tiles * p.m_tiles;
    int ranks = 1;
    while (ranks < 8 && base * ranks < target && stages / (ranks * 2) >= 2) ranks *= 2;
    p.spr = cdiv(stages, ranks);
    p.ranks = ranks;
    return p;
}

template <int NJ, bool ZTABLE, int GPS, int WN>
int launch_one(const W4Params& p, const Plan& pl, cudaStream_t st) {
    using L = Layout<NJ, WN, GPS>;
    auto kernel = w4a16_stream_kernel<NJ, ZTABLE, GPS, WN>;
    static bool configured[64] = {};                   // per instantiation and device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LQ2_ERR_CUDA;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES) != cudaSuccess)
            return LQ2_ERR_CUDA;
        configured[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.n_tiles, pl.ranks, pl.m_tiles);
    cfg.blockDim = dim3(32 * WN);
    cfg.dynamicSmemBytes = L::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = pl.ranks;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? LQ2_OK : LQ2_ERR_CUDA;
}

template <int NJ, bool ZTABLE, int GPS>
int launch_wn(const W4Params& p, const Plan& pl, cudaStream_t st) {
    return pl.wn == 4 ? launch_one<NJ, ZTABLE, GPS, 4>(p, pl, st) : launch_one<NJ, ZTABLE, GPS, 2>(p, pl, st);
}

template <int NJ, bool ZTABLE>
int launch_gps(const W4Params& p, const Plan& pl, cudaStream_t st) {
    const int gps = p.group >= 128 ? 1 : 128 / p.group;
    if (gps == 1) return launch_wn<NJ, ZTABLE, 1>(p, pl, st);
    if (gps == 2) return launch_wn<NJ, ZTABLE, 2>(p, pl, st);
    return launch_wn<NJ, ZTABLE, 4>(p, pl, st);
}

template <int NJ>
int launch_z(const W4Params& p, const Plan& pl, cudaStream_t st) {
    return p.zeros ? launch_gps<NJ, true>(p, pl, st) : launch_gps<NJ, false>(p, pl, st);
}

}  // namespace

// The cluster reduction keeps split-K partials on chip; no global scratch is needed.
size_t w4a16_stream_workspace_bytes(int, int, int) { return 0; }

int w4a16_stream_launch(const __half* x, int64_t ldx, const int32_t* packed, const __half* scales,
                        const __half* zeros, __half* y, int m, int n, int k, int group,
                        void*, size_t, cudaStream_t st) {
    const Plan pl = make_plan(m, n, k);
    if (pl.m_tiles > 65535) return LQ2_ERR_SHAPE;
    W4Params p;
    p.x = x; p.ldx = ldx; p.packed = packed; p.scales = scales; p.zeros = zeros; p.y = y;
    p.m = m; p.n = n; p.k = k; p.group = group;
    p.stages_per_rank = pl.spr;
    switch (pl.nj) {
        case 1: return launch_z<1>(p, pl, st);
        case 2: return launch_z<2>(p, pl, st);
        case 4: return launch_z<4>(p, pl, st);
        default: return launch_z<8>(p, pl, st);
    }
}

}  // namespace lq2
