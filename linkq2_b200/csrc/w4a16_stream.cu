// W4A16 linear for small M (decode GEMV, batched decode, 16-position verify):
// a weight-streaming kernel bounded by HBM bandwidth.
//
// Replaces the GEMV and split-K Triton routes of the reference
// (qslab/kernels/gemlite/triton_kernels/gemv_revsplitK_A16fWnO16f_int32packing.py:155-384,
//  gemm_splitK_A16fWnO16f_int32packing.py:199-412) behind the same buffers:
//   packed [K/8, N] int32 (n fastest; nibble j of word (k8, n) is k = 8*k8 + j),
//   scales / zeros [K/group, N] fp16.
//
// Data movement.  A warp owns 32 output columns.  Lane (g, t) = (lane / 4, lane % 4)
// reads one 128-bit word quad per step: packed[k8 = 4*step + t][n0 .. n0+3] with
// n0 = 32*warp_tile + 4*g, so every warp-level load instruction covers four
// 128-byte rows, and eight warps of a CTA cover 1 KiB contiguous per row.  The
// nibbles are unpacked in registers and fed to the warp-level tensor-core op
// m16n8k16 used as a dot-product engine: the MMA's 16 "rows" are output columns
// (two per lane-group), its 16 k-slots are the eight nibbles of lane t's words
// in an order chosen so that unpacking needs one shift per word, and its 8
// "columns" are activation rows.  The four lanes of a group hold different k,
// so the MMA performs the cross-lane reduction itself; nothing is shuffled.
//
// For M <= 8 the group scale is applied after the group's integer dot product:
//   y += s * (sum_k (u - 8) x_k  -  (z - 8) * sum_k x_k)
// with the activation sum produced by one extra MMA against a fragment of ones.
// This keeps the per-weight work at ~1 ALU op.  For 8 < M <= 64 weights are
// dequantised to fp16 exactly as the reference does, (u - z) * s rounded once
// (triton_kernels/utils.py:66-71), and accumulated in fp32.
//
// Split-K: grid.y CTAs share a column tile.  Each writes an fp32 partial to the
// workspace, takes a ticket, and the last one to arrive adds the partials in
// split order (so the result does not depend on arrival order), writes fp16 and
// resets the ticket counter for the next call.
#include "common.cuh"

namespace lq2 {

namespace {

constexpr int kStageK = 128;                     // k per pipeline stage
constexpr int kXsRowBytes = kStageK * 2 + 64;    // +64: conflict-free 128-bit fragment loads
constexpr int kThreads = 256;
constexpr int kTileN = 256;                      // 8 warps x 32 columns
constexpr int kCounterInts = 4096;

struct W4Params {
    const __half* x;
    int64_t ldx;
    const int32_t* packed;
    const __half* scales;
    const __half* zeros;
    __half* y;
    int m, n, k, group;
    int splits, stages_per_split;
    float* partial;
    int* counters;
};

struct Plan {
    int nj, m_tiles, n_tiles, splits, sps;
};

Plan make_plan(int m, int n, int k) {
    Plan p;
    p.nj = m <= 8 ? 1 : (m <= 16 ? 2 : (m <= 32 ? 4 : 8));
    p.m_tiles = cdiv(m, 8 * p.nj);
    p.n_tiles = cdiv(n, kTileN);
    const int stages = cdiv(k, kStageK);
    const int base = p.n_tiles * p.m_tiles;
    const int slots = kNumSMs * (p.nj <= 2 ? 2 : 1);
    int splits = base >= slots ? 1 : slots / base;
    if (splits > stages / 2) splits = stages / 2 > 0 ? stages / 2 : 1;
    const int64_t cap = (int64_t(32) << 20) / (int64_t(m) * n * 4);
    if (splits > cap) splits = cap > 0 ? int(cap) : 1;
    if (splits < 1) splits = 1;
    p.sps = cdiv(stages, splits);
    p.splits = cdiv(stages, p.sps);
    return p;
}

__device__ __forceinline__ uint32_t bcast_half(uint2 v, int idx) {
    // half #idx of the four halves in v, replicated into both lanes of a half2
    const uint32_t w = idx < 2 ? v.x : v.y;
    return __byte_perm(w, w, (idx & 1) ? 0x3232 : 0x1010);
}

__device__ __forceinline__ float half_at(uint2 v, int idx) {
    const uint32_t w = idx < 2 ? v.x : v.y;
    return __half2float(__ushort_as_half((unsigned short)((idx & 1) ? (w >> 16) : (w & 0xffff))));
}

template <int NJ, bool ZTABLE, int GPS>
__global__ void __launch_bounds__(kThreads, (NJ <= 2 ? 2 : 1))
w4a16_stream_kernel(const W4Params p) {
    constexpr bool SCALE_AFTER = (NJ == 1);
    constexpr int MT = 8 * NJ;
    constexpr int XCH = (MT * 16 + kThreads - 1) / kThreads;
    constexpr int STEPS_PER_GROUP = 4 / GPS;     // 32-k steps per scale group inside a stage

    __shared__ __align__(16) unsigned char xs[2][MT][kXsRowBytes];
    __shared__ int s_ticket;

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int m0 = blockIdx.z * MT;
    const int rows = min(MT, p.m - m0);
    const int nb = blockIdx.x * kTileN + warp * 32;
    const bool n_ok = nb < p.n;
    const int n0 = nb + 4 * g;
    const int k8_total = p.k >> 3;
    const int total_stages = (p.k + kStageK - 1) / kStageK;
    const int s0 = blockIdx.y * p.stages_per_split;
    const int s1 = min(total_stages, s0 + p.stages_per_split);
    const int groups_total = p.k / p.group;

    for (int i = tid; i < int(sizeof(xs) / 16); i += kThreads)
        reinterpret_cast<uint4*>(&xs[0][0][0])[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();

    uint4 xr[XCH];
    auto load_x = [&](int s) {
#pragma unroll
        for (int c = 0; c < XCH; ++c) {
            const int id = tid + c * kThreads;
            const int row = id >> 4, kc = id & 15;
            const int kk = s * kStageK + kc * 8;
            xr[c] = make_uint4(0, 0, 0, 0);
            if (row < rows && kk < p.k)
                xr[c] = *reinterpret_cast<const uint4*>(p.x + int64_t(m0 + row) * p.ldx + kk);
        }
    };
    auto store_x = [&](int buf) {
#pragma unroll
        for (int c = 0; c < XCH; ++c) {
            const int id = tid + c * kThreads;
            const int row = id >> 4, kc = id & 15;
            if (id < MT * 16) {
                // halves x0..x7 -> x0 x4 x1 x5 x2 x6 x3 x7 (the k-slot order of the MMA fragments)
                uint4 o;
                o.x = __byte_perm(xr[c].x, xr[c].z, 0x5410);
                o.y = __byte_perm(xr[c].x, xr[c].z, 0x7632);
                o.z = __byte_perm(xr[c].y, xr[c].w, 0x5410);
                o.w = __byte_perm(xr[c].y, xr[c].w, 0x7632);
                *reinterpret_cast<uint4*>(&xs[buf][row][kc * 16]) = o;
            }
        }
    };
    auto load_w = [&](int s, uint4 (&w)[4]) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const int k8 = s * 16 + kk * 4 + t;
            w[kk] = make_uint4(0, 0, 0, 0);
            if (n_ok && k8 < k8_total) w[kk] = ldg_stream_u4(p.packed + int64_t(k8) * p.n + n0);
        }
    };
    auto load_s = [&](int s, uint2 (&sc)[GPS], uint2 (&zc)[GPS]) {
#pragma unroll
        for (int q = 0; q < GPS; ++q) {
            int gi = (GPS == 1) ? (s * kStageK) / p.group : s * GPS + q;
            gi = min(gi, groups_total - 1);
            sc[q] = make_uint2(0, 0);
            zc[q] = make_uint2(0, 0);
            if (n_ok) {
                sc[q] = ldg_stream_u2(p.scales + int64_t(gi) * p.n + n0);
                if (ZTABLE) zc[q] = ldg_stream_u2(p.zeros + int64_t(gi) * p.n + n0);
            }
        }
    };

    float acc[2][NJ][4];
    float gacc[SCALE_AFTER ? 2 : 1][SCALE_AFTER ? NJ : 1][4];
    float xsum[SCALE_AFTER ? NJ : 1][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;
    if (SCALE_AFTER) {
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) gacc[i][0][c] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) xsum[0][c] = 0.f;
    }

    const __half2 k1032 = __floats2half2_rn(1032.f, 1032.f);
    const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
    const __half2 km72 = __floats2half2_rn(-72.f, -72.f);
    const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
    const __half2 k64 = __floats2half2_rn(64.f, 64.f);
    constexpr uint32_t kOnes = 0x3C003C00u;

    uint4 wq[4], wn[4];
    uint2 sc[GPS], zc[GPS], scn[GPS], zcn[GPS];

    if (s0 < s1) {
        load_w(s0, wq);
        load_s(s0, sc, zc);
        load_x(s0);
        store_x(0);
    }
    __syncthreads();

    for (int s = s0; s < s1; ++s) {
        const int buf = (s - s0) & 1;
        const bool has_next = s + 1 < s1;
        if (has_next) {
            load_w(s + 1, wn);
            load_s(s + 1, scn, zcn);
            load_x(s + 1);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t wv[4] = {wq[kk].x, wq[kk].y, wq[kk].z, wq[kk].w};
            uint4 xb[NJ];
#pragma unroll
            for (int j = 0; j < NJ; ++j)
                xb[j] = *reinterpret_cast<const uint4*>(&xs[buf][8 * j + g][(kk * 4 + t) * 16]);
            const int gq = kk / STEPS_PER_GROUP;
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                __half2 s_a, s_b, zlo_a, zlo_b, zhi_a, zhi_b;
                if (!SCALE_AFTER) {
                    s_a = u32_as_h2(bcast_half(sc[gq], 2 * i));
                    s_b = u32_as_h2(bcast_half(sc[gq], 2 * i + 1));
                    if (ZTABLE) {
                        const __half2 z_a = u32_as_h2(bcast_half(zc[gq], 2 * i));
                        const __half2 z_b = u32_as_h2(bcast_half(zc[gq], 2 * i + 1));
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
                        if (SCALE_AFTER) mma_m16n8k16(gacc[i][j], a0, a1, a2, a3, b0, b1);
                        else mma_m16n8k16(acc[i][j], a0, a1, a2, a3, b0, b1);
                    }
                }
            }
            if (SCALE_AFTER) {
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
                        const float sa = half_at(sc[gq], 2 * i), sb = half_at(sc[gq], 2 * i + 1);
                        float za = 0.f, zb = 0.f;
                        if (ZTABLE) {
                            za = half_at(zc[gq], 2 * i) - 8.f;
                            zb = half_at(zc[gq], 2 * i + 1) - 8.f;
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
        if (has_next) store_x(buf ^ 1);
        __syncthreads();
        if (has_next) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) wq[kk] = wn[kk];
#pragma unroll
            for (int q = 0; q < GPS; ++q) {
                sc[q] = scn[q];
                zc[q] = zcn[q];
            }
        }
    }

    // ---- write-out.  Lane (g, t) owns columns n0..n0+3 of rows m0 + 8j + 2t (+1).
    const int splits = p.splits;
    if (splits == 1) {
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

    if (n_ok) {
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int m = m0 + 8 * j + 2 * t + r;
                if (m < p.m) {
                    float4 v = make_float4(acc[0][j][r], acc[0][j][2 + r], acc[1][j][r], acc[1][j][2 + r]);
                    __stcg(reinterpret_cast<float4*>(p.partial + (int64_t(blockIdx.y) * p.m + m) * p.n + n0), v);
                }
            }
        }
    }
    __threadfence();
    __syncthreads();
    int* counter = p.counters + blockIdx.z * gridDim.x + blockIdx.x;
    if (tid == 0) s_ticket = atomicAdd(counter, 1);
    __syncthreads();
    if (s_ticket != splits - 1) return;
    __threadfence();
    if (n_ok) {
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int m = m0 + 8 * j + 2 * t + r;
                if (m < p.m) {
                    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int sp = 0; sp < splits; ++sp) {
                        const float4 v = __ldcg(reinterpret_cast<const float4*>(
                            p.partial + (int64_t(sp) * p.m + m) * p.n + n0));
                        sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
                    }
                    const __half2 lo = __floats2half2_rn(sum.x, sum.y);
                    const __half2 hi = __floats2half2_rn(sum.z, sum.w);
                    *reinterpret_cast<uint2*>(p.y + int64_t(m) * p.n + n0) =
                        make_uint2(h2_as_u32(lo), h2_as_u32(hi));
                }
            }
        }
    }
    if (tid == 0) *counter = 0;
}

template <int NJ, bool ZTABLE>
int launch_gps(const W4Params& p, dim3 grid, cudaStream_t st) {
    const int gps = p.group >= 128 ? 1 : 128 / p.group;
    if (gps == 1) w4a16_stream_kernel<NJ, ZTABLE, 1><<<grid, kThreads, 0, st>>>(p);
    else if (gps == 2) w4a16_stream_kernel<NJ, ZTABLE, 2><<<grid, kThreads, 0, st>>>(p);
    else w4a16_stream_kernel<NJ, ZTABLE, 4><<<grid, kThreads, 0, st>>>(p);
    return check_launch();
}

template <int NJ>
int launch_z(const W4Params& p, dim3 grid, cudaStream_t st) {
    return p.zeros ? launch_gps<NJ, true>(p, grid, st) : launch_gps<NJ, false>(p, grid, st);
}

}  // namespace

size_t w4a16_stream_workspace_bytes(int m, int n, int k) {
    const Plan pl = make_plan(m, n, k);
    size_t bytes = size_t(kCounterInts) * sizeof(int);
    if (pl.splits > 1) bytes += size_t(pl.splits) * m * n * sizeof(float);
    return bytes;
}

int w4a16_stream_launch(const __half* x, int64_t ldx, const int32_t* packed, const __half* scales,
                        const __half* zeros, __half* y, int m, int n, int k, int group,
                        void* workspace, size_t workspace_bytes, cudaStream_t st) {
    const Plan pl = make_plan(m, n, k);
    if (pl.n_tiles * pl.m_tiles > kCounterInts) return LQ2_ERR_SHAPE;
    if (workspace_bytes < w4a16_stream_workspace_bytes(m, n, k) || !workspace) return LQ2_ERR_WORKSPACE;
    W4Params p;
    p.x = x; p.ldx = ldx; p.packed = packed; p.scales = scales; p.zeros = zeros; p.y = y;
    p.m = m; p.n = n; p.k = k; p.group = group;
    p.splits = pl.splits; p.stages_per_split = pl.sps;
    p.counters = reinterpret_cast<int*>(workspace);
    p.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + size_t(kCounterInts) * sizeof(int));
    dim3 grid(pl.n_tiles, pl.splits, pl.m_tiles);
    switch (pl.nj) {
        case 1: return launch_z<1>(p, grid, st);
        case 2: return launch_z<2>(p, grid, st);
        case 4: return launch_z<4>(p, grid, st);
        default: return launch_z<8>(p, grid, st);
    }
}

}  // namespace lq2
