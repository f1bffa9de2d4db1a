// W4A16 linear for small M (decode GEMV, batched decode, 16-position verify):
// a weight-streaming kernel bounded by HBM bandwidth.
//
// Replaces the GEMV and split-K Triton routes of the reference
// (qslab/kernels/gemlite/triton_kernels/gemv_revsplitK_A16fWnO16f_int32packing.py:155-384,
//  gemm_splitK_A16fWnO16f_int32packing.py:199-412) behind the same buffers:
//   packed [K/8, N] int32 (n fastest; nibble j of word (k8, n) is k = 8*k8 + j),
//   scales / zeros [K/group, N] fp16.
//
// Data movement.  A CTA owns 32*WN output columns and a contiguous range of K.
// One producer warp keeps a ring of STAGES shared-memory buffers (128 k each)
// full with tiled TMA loads (cp.async.bulk.tensor, 128-byte swizzle, no
// cluster-wide broadcast) of packed words, activations, scales and zero points, signalled
// through mbarriers; WN consumer warps wait on a stage, use it and hand it back.
// Rows or columns past the end of a tensor are zero-filled by the TMA unit.  The
// bytes in flight per SM are set by the ring depth, and the main loop has no
// CTA-wide barrier.  Consumer lane (g, t) = (lane / 4, lane % 4) reads one
// 128-bit word quad per step, packed[k8 row of (step, t)][n0 .. n0+3] with
// n0 = 32*warp + 4*g, at its swizzled position; the rows a step uses are chosen
// so that these reads are free of bank conflicts.
//
// Arithmetic.  The nibbles go to the warp-level tensor-core op m16n8k16, used as
// an fp32-accumulating dot-product engine, without any conversion: a nibble u
// masked in place is the fp16 subnormal u * 2^-24 (even nibbles) or 16u * 2^-24
// (odd nibbles, whose activations are divided by 16 to compensate), which the
// tensor core multiplies exactly.  The MMA's 16 "rows" are output columns (two
// per lane group), its 16 k-slots the eight nibbles of lane t's words in the
// order the masks produce (the activation fragment is permuted to match), its 8
// "columns" activation rows.  The four lanes of a group hold different k, so the
// MMA performs the cross-lane reduction itself.  Per quantization group
//   y += s * (2^24 * sum_k u' x_k  -  z * sum_k x_k),
// the activation sum coming from one extra MMA against a constant fragment.
// This equals sum_k ((u - z) * s) x_k of the reference's dequantisation
// (triton_kernels/utils.py:66-71) evaluated in fp32, for any fp16 zero point;
// the only rounding beyond fp32 accumulation is x/16 for |x| < 2^-10.
//
// Split-K.  The CTAs that share a column tile form a thread-block cluster along
// grid.y.  Rank q of the cluster owns a slice of the tile's columns; every rank
// writes its fp32 partial sums for that slice from registers straight into q's
// receive area (distributed shared memory stores), one cluster barrier follows, and
// q adds the parts in rank order (so the result does not depend on timing) and
// writes fp16.  No global scratch, no atomics.
#include <cooperative_groups.h>
#include <cuda.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lq2 {

namespace {

constexpr int kStageK = 128;                     // k per pipeline stage

struct W4Params {
    const __half* x;
    int64_t ldx;
    const int32_t* packed;
    const __half* scales;
    const __half* zeros;
    __half* y;
    int m, n, k, group;
    int stages_per_rank;
    int early_weights;    // request weight bytes before the previous kernel of the stream has finished
    int silu;             // columns are interleaved [4 gate | 4 up]: write silu(gate) * up, N / 2 wide
};

// ---- mbarrier / bulk-copy primitives (shared::cta addresses as 32-bit values)
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n.reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// Number of waits that gave up (see mbar_wait); stays 0 in a healthy run.
__device__ unsigned int g_lq2_w4_wait_timeouts = 0;
// Bounded wait: try_wait suspends the thread for a hardware time slice per call;
// after kMaxWaitPolls unsuccessful polls the wait is abandoned, the give-up is
// counted in g_lq2_w4_wait_timeouts and the kernel runs on to its end (its
// output is then wrong, but the GPU is not left spinning).
constexpr int kMaxWaitPolls = 1 << 22;
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < kMaxWaitPolls; ++i)
        if (mbar_try_wait(bar, parity)) return;
    atomicAdd(&g_lq2_w4_wait_timeouts, 1u);
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(map) : "memory");
}
// 2-D tiled TMA load (one CTA is the only receiver): box at element coordinates (c0 = innermost, c1) -> shared memory
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
        ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar) : "memory");
}

__device__ __forceinline__ float half_at(uint2 v, int idx) {
    const uint32_t w = idx < 2 ? v.x : v.y;
    return __half2float(__ushort_as_half((unsigned short)((idx & 1) ? (w >> 16) : (w & 0xffff))));
}

template <int NJ, int WN, int GPS>
struct Layout {
    static constexpr int MT = 8 * NJ;
    static constexpr int TN = 32 * WN;
    static constexpr int NJW = NJ < 2 ? NJ : 2;                 // 8-row activation blocks per consumer warp
    static constexpr int JS = NJ / NJW;                         // consumer warps that share a slab, splitting the rows
    static constexpr int CONSUMERS = WN * JS;
    static constexpr int THREADS = 32 * (CONSUMERS + 1);
    static constexpr int SLAB_BYTES = 16 * 128;                 // one warp's 16 rows x 32 columns, 128B-swizzled
    static constexpr int W_BYTES = WN * SLAB_BYTES;
    static constexpr int XBOX_BYTES = MT * 128;                 // MT rows x 64 k, 128B-swizzled
    static constexpr int X_BYTES = 2 * XBOX_BYTES;
    static constexpr int S_BYTES = GPS * TN * 2;
    static constexpr int TX_BYTES = W_BYTES + X_BYTES;          // + S_BYTES (x2 with zero points)
    static constexpr int STAGE_BYTES = (W_BYTES + X_BYTES + 2 * S_BYTES + 1023) / 1024 * 1024;
    static constexpr int STAGES = NJ <= 2 ? 4 : 3;
    static constexpr int RED_BYTES = MT * TN * 4;               // receive area of the split-K reduction
    static constexpr int RING_BYTES = STAGES * STAGE_BYTES;
    static constexpr int RECV_OFF = RING_BYTES;                 // never aliased with the ring: peers write into it
    static constexpr int DATA_BYTES = RING_BYTES + RED_BYTES;
    static constexpr int SMEM_BYTES = 1024 + DATA_BYTES + 2 * STAGES * 8;   // alignment slack + mbarriers
};

// Warps 0..CONSUMERS-1 consume: warp w works on column slab w % WN and on the
// activation rows of block (w / WN) * 16 .. +15 (two 8-row MMA column blocks), so a
// 32-row batch keeps eight consumer warps busy; the last warp is the producer that
// keeps the ring full with TMA loads.  No CTA-wide barrier inside the main loop.
template <int NJ, bool ZTABLE, int GPS, int WN>
__global__ void __launch_bounds__(Layout<NJ, WN, GPS>::THREADS, (NJ <= 2 ? 4 : (NJ == 4 ? 3 : 1))) w4a16_stream_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                    const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                    const W4Params p) {
    using L = Layout<NJ, WN, GPS>;
    constexpr int MT = L::MT, TN = L::TN, STAGES = L::STAGES, CONSUMERS = L::CONSUMERS, NJW = L::NJW;
    constexpr int STEPS_PER_GROUP = 4 / GPS;
    constexpr int STEPS = 4;                                 // 32-k steps of a stage
    // k8 row (and activation chunk) that lane t uses in step kk.  Rows 2t + (kk & 1) of an
    // 8-row block make the swizzled 128-bit reads conflict-free; with four groups per
    // stage a step must stay inside 4 consecutive rows instead.
    constexpr bool INTERLEAVE = GPS <= 2;

    pdl_launch_dependents();
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);   // swizzle atoms are 1 KiB
    const uint32_t bars = smem_u32(smem + L::DATA_BYTES);    // full[STAGES], empty[STAGES]

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    if (threadIdx.x == 0) {                  // the tensor maps' descriptors are on their way before the first copy needs them
        prefetch_tensormap(&map_w);
        prefetch_tensormap(&map_x);
        prefetch_tensormap(&map_s);
        prefetch_tensormap(&map_z);
    }
    const int m0 = blockIdx.z * MT;
    const int rows = min(MT, p.m - m0);
    const int tile_n0 = blockIdx.x * TN;
    const int total_stages = (p.k + kStageK - 1) / kStageK;
    const int ranks = gridDim.y, rank = blockIdx.y;
    const int s0 = min(total_stages, rank * p.stages_per_rank);
    const int s1 = min(total_stages, s0 + p.stages_per_rank);
    const int my_stages = s1 - s0;

    if (tid == 0) {
        for (int i = 0; i < STAGES; ++i) {
            mbar_init(bars + 8 * i, 1);                       // full: the producer's arrive + bytes
            mbar_init(bars + 8 * (STAGES + i), CONSUMERS);    // empty: one arrive per consumer warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    // first half of a cluster barrier: by the time the epilogue waits for it, every CTA of
    // the cluster is known to be running, which remote shared-memory stores require
    if (ranks > 1) asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");

    float acc[2][NJW][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < NJW; ++j)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.f;

    const int slab = warp % WN, jpart = warp / WN;           // first activation block of this warp: jpart * NJW
    if (warp == CONSUMERS) {
        // ------------------------------------------------------------ producer
        // Out-of-range rows and columns are zero-filled by the TMA unit and still count
        // their full box size, so the expected byte count of a stage is a constant.
        auto load_weights = [&](int it) {
            const int slot = it % STAGES, s = s0 + it;
            const uint32_t full = bars + 8 * slot;
            const uint32_t base = smem_u32(smem + slot * L::STAGE_BYTES);
            mbar_arrive_expect_tx(full, L::TX_BYTES + L::S_BYTES * (ZTABLE ? 2 : 1));
#pragma unroll
            for (int w = 0; w < WN; ++w)
                tma_load_2d(base + w * L::SLAB_BYTES, &map_w, tile_n0 + 32 * w, s * 16, full);
            const int gi = (GPS == 1) ? (s * kStageK) / p.group : s * GPS;
            tma_load_2d(base + L::W_BYTES + L::X_BYTES, &map_s, tile_n0, gi, full);
            if (ZTABLE) tma_load_2d(base + L::W_BYTES + L::X_BYTES + L::S_BYTES, &map_z, tile_n0, gi, full);
        };
        auto load_activations = [&](int it) {
            const int slot = it % STAGES, s = s0 + it;
            const uint32_t full = bars + 8 * slot;
            const uint32_t base = smem_u32(smem + slot * L::STAGE_BYTES);
            tma_load_2d(base + L::W_BYTES, &map_x, s * kStageK, m0, full);
            tma_load_2d(base + L::W_BYTES + L::XBOX_BYTES, &map_x, s * kStageK + 64, m0, full);
        };
        // When the caller has declared the weights constant, the first ring of weight bytes
        // is requested before the previous kernel of the stream has finished; the
        // activations, which that kernel may still be writing, only after pdl_wait().
        const int ahead = min(my_stages, STAGES);
        if (!p.early_weights) pdl_wait();
        if (lane == 0)
            for (int it = 0; it < ahead; ++it) load_weights(it);
        if (p.early_weights) pdl_wait();
        if (lane == 0)
            for (int it = 0; it < ahead; ++it) load_activations(it);
        __syncwarp();
        for (int it = ahead; it < my_stages; ++it) {
            mbar_wait(bars + 8 * (STAGES + it % STAGES), ((it / STAGES) - 1) & 1);
            if (lane == 0) {
                load_weights(it);
                load_activations(it);
            }
            __syncwarp();
        }
    } else {
        // ------------------------------------------------------------ consumers
        pdl_wait();
        float gacc[2][NJW][4];
        float xsum[NJW][4];
#pragma unroll
        for (int j = 0; j < NJW; ++j) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                gacc[0][j][c] = 0.f;
                gacc[1][j][c] = 0.f;
                xsum[j][c] = 0.f;
            }
        }
        const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
        constexpr uint32_t kOnes = 0x3C003C00u;
        constexpr float kTwo24 = 16777216.f;
        // unrolled over the ring: the stage slot and its addresses are compile-time constants
        uint32_t ring_phase = 0;                              // (it / STAGES) & 1
        for (int it0 = 0; it0 < my_stages; it0 += STAGES, ring_phase ^= 1u) {
#pragma unroll
          for (int slot = 0; slot < STAGES; ++slot) {
            if (it0 + slot >= my_stages) break;
            mbar_wait(bars + 8 * slot, ring_phase);
            const unsigned char* base = smem + slot * L::STAGE_BYTES;
            const unsigned char* wsm = base + slab * L::SLAB_BYTES;
            const unsigned char* xsm = base + L::W_BYTES;
            const unsigned char* ssm = xsm + L::X_BYTES + slab * 64 + g * 8;
#pragma unroll
            for (int kk = 0; kk < STEPS; ++kk) {
                const int row = INTERLEAVE ? 8 * (kk >> 1) + 2 * t + (kk & 1) : 4 * kk + t;
                // 128B swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)
                const uint4 wq = *reinterpret_cast<const uint4*>(wsm + row * 128 + ((g ^ (row & 7)) << 4));
                const uint32_t wv[4] = {wq.x, wq.y, wq.z, wq.w};
                uint4 xb[NJW];
#pragma unroll
                for (int j = 0; j < NJW; ++j) {
                    const uint4 r = *reinterpret_cast<const uint4*>(
                        xsm + (row >> 3) * L::XBOX_BYTES + (8 * (jpart * NJW + j) + g) * 128 + (((row & 7) ^ g) << 4));
                    // halves x0..x7 -> {x0,x4} {x1,x5}/16 {x2,x6} {x3,x7}/16: the k-slot order of the A
                    // fragments; odd nibbles enter A multiplied by 16 (no shift), so their x is divided by 16
                    xb[j].x = __byte_perm(r.x, r.z, 0x5410);
                    xb[j].y = h2_as_u32(__hmul2(u32_as_h2(__byte_perm(r.x, r.z, 0x7632)), k16th));
                    xb[j].z = __byte_perm(r.y, r.w, 0x5410);
                    xb[j].w = h2_as_u32(__hmul2(u32_as_h2(__byte_perm(r.y, r.w, 0x7632)), k16th));
                }
#pragma unroll
                for (int i = 0; i < 2; ++i) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        // nibbles as fp16 subnormals: u * 2^-24 (even nibbles) and 16u * 2^-24 (odd nibbles)
                        const uint32_t wa = wv[2 * i] >> (8 * h);
                        const uint32_t wb = wv[2 * i + 1] >> (8 * h);
                        const uint32_t a0 = wa & 0x000f000fu, a1 = wb & 0x000f000fu;
                        const uint32_t a2 = wa & 0x00f000f0u, a3 = wb & 0x00f000f0u;
#pragma unroll
                        for (int j = 0; j < NJW; ++j)
                            mma_m16n8k16(gacc[i][j], a0, a1, a2, a3, h ? xb[j].z : xb[j].x, h ? xb[j].w : xb[j].y);
                    }
                }
#pragma unroll
                for (int j = 0; j < NJW; ++j) {
                    // sum of the step's activations (undoing the 1/16 on the odd slots with 16.0 in A)
                    constexpr uint32_t k16s = 0x4C004C00u;
                    mma_m16n8k16(xsum[j], kOnes, kOnes, k16s, k16s, xb[j].x, xb[j].y);
                    mma_m16n8k16(xsum[j], kOnes, kOnes, k16s, k16s, xb[j].z, xb[j].w);
                }
                // end of a scale group, or of this warp's share of one (the scale then multiplies a
                // partial sum, which is the same by linearity)
                if ((kk + 1) % (STEPS_PER_GROUP < STEPS ? STEPS_PER_GROUP : STEPS) == 0) {
                    const int gq = kk / STEPS_PER_GROUP;
                    const uint2 sc = *reinterpret_cast<const uint2*>(ssm + gq * TN * 2);
                    uint2 zc = make_uint2(0x48004800u, 0x48004800u);           // 8.0 x4
                    if (ZTABLE) zc = *reinterpret_cast<const uint2*>(ssm + L::S_BYTES + gq * TN * 2);
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        // s * sum_k (u - z) x = (s * 2^24) * gacc - (s * z) * xsum
                        const float sa = half_at(sc, 2 * i), sb = half_at(sc, 2 * i + 1);
                        const float za = -sa * half_at(zc, 2 * i), zb = -sb * half_at(zc, 2 * i + 1);
                        const float ta = sa * kTwo24, tb = sb * kTwo24;
#pragma unroll
                        for (int j = 0; j < NJW; ++j) {
                            acc[i][j][0] = fmaf(ta, gacc[i][j][0], fmaf(za, xsum[j][0], acc[i][j][0]));
                            acc[i][j][1] = fmaf(ta, gacc[i][j][1], fmaf(za, xsum[j][1], acc[i][j][1]));
                            acc[i][j][2] = fmaf(tb, gacc[i][j][2], fmaf(zb, xsum[j][0], acc[i][j][2]));
                            acc[i][j][3] = fmaf(tb, gacc[i][j][3], fmaf(zb, xsum[j][1], acc[i][j][3]));
#pragma unroll
                            for (int c = 0; c < 4; ++c) gacc[i][j][c] = 0.f;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < NJW; ++j)
#pragma unroll
                        for (int c = 0; c < 4; ++c) xsum[j][c] = 0.f;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bars + 8 * (STAGES + slot));
          }
        }
    }

    const int nb = tile_n0 + slab * 32;
    const bool n_ok = warp < CONSUMERS && nb < p.n;
    const int n0 = nb + 4 * g;

    // ---- write-out.  Consumer lane (g, t) owns columns n0..n0+3 of rows m0 + 8j + 2t (+1).
    if (ranks == 1) {
        if (p.silu) {
            // lane groups with even g hold four gate channels, their neighbours (g + 1) the matching
            // four up channels: fetch those with a shuffle, then the even groups write
            if (warp < CONSUMERS) {
#pragma unroll
                for (int j = 0; j < NJW; ++j) {
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const float4 mine = make_float4(acc[0][j][r], acc[0][j][2 + r], acc[1][j][r], acc[1][j][2 + r]);
                        float4 up;
                        up.x = __shfl_xor_sync(0xffffffffu, mine.x, 4);
                        up.y = __shfl_xor_sync(0xffffffffu, mine.y, 4);
                        up.z = __shfl_xor_sync(0xffffffffu, mine.z, 4);
                        up.w = __shfl_xor_sync(0xffffffffu, mine.w, 4);
                        const int m = m0 + 8 * (jpart * NJW + j) + 2 * t + r;
                        if (n_ok && (g & 1) == 0 && m < p.m)
                            *reinterpret_cast<uint2*>(p.y + int64_t(m) * (p.n / 2) + n0 / 2) = silu_mul_quad(mine, up);
                    }
                }
            }
            return;
        }
        if (n_ok) {
#pragma unroll
            for (int j = 0; j < NJW; ++j) {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const int m = m0 + 8 * (jpart * NJW + j) + 2 * t + r;
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

    // ---- split-K reduction.  Rank q of the cluster owns columns [q * W, (q + 1) * W) of the tile.
    // Every rank writes its partial sums for those columns straight from registers into q's
    // receive area (remote shared memory), one cluster barrier follows, and q adds the ranks'
    // parts in rank order.  Nobody reads remote memory after the barrier, so a CTA may leave as
    // soon as it has written its slice.
    cg::cluster_group cluster = cg::this_cluster();
    const int W = TN / ranks;
    float* recv = reinterpret_cast<float*>(smem + L::RECV_OFF);       // [ranks][MT][W]
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");   // all CTAs of the cluster are running
    if (warp < CONSUMERS) {
        const int col = slab * 32 + 4 * g;
        const int dest = col / W, c = col - dest * W;
        float* dst = cluster.map_shared_rank(recv, dest) + size_t(rank) * MT * W + c;
#pragma unroll
        for (int j = 0; j < NJW; ++j) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int ml = 8 * (jpart * NJW + j) + 2 * t + r;
                *reinterpret_cast<float4*>(dst + ml * W) =
                    make_float4(acc[0][j][r], acc[0][j][2 + r], acc[1][j][r], acc[1][j][2 + r]);
            }
        }
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
    auto slice_sum = [&](int ml, int col) {
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < ranks; ++q) {
            const float4 v = *reinterpret_cast<const float4*>(recv + (size_t(q) * MT + ml) * W + col);
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
        }
        return sum;
    };
    if (p.silu) {
        const int octs = W / 8;                            // [4 gate | 4 up] blocks of my slice
        for (int e = tid; e < rows * octs; e += L::THREADS) {
            const int ml = e / octs, col = (e - ml * octs) * 8;
            const int nn = tile_n0 + rank * W + col;
            if (nn < p.n)
                *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * (p.n / 2) + nn / 2) =
                    silu_mul_quad(slice_sum(ml, col), slice_sum(ml, col + 4));
        }
    } else {
        const int quads = W / 4;
        for (int e = tid; e < rows * quads; e += L::THREADS) {
            const int ml = e / quads, col = (e - ml * quads) * 4;
            const float4 sum = slice_sum(ml, col);
            const int nn = tile_n0 + rank * W + col;
            if (nn < p.n) {
                const __half2 lo = __floats2half2_rn(sum.x, sum.y);
                const __half2 hi = __floats2half2_rn(sum.z, sum.w);
                *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * p.n + nn) = make_uint2(h2_as_u32(lo), h2_as_u32(hi));
            }
        }
    }
}

struct Plan {
    int nj, wn, m_tiles, n_tiles, ranks, spr;
};

// Column-tile width and cluster size from shapes only.  Streaming is fastest when
// every CTA is resident at once (up to four per SM) and each one streams a long
// K range, so: 128-column tiles unless even the largest cluster leaves SMs
// without a CTA, and the largest power-of-two cluster (K split) that keeps the
// grid within one resident wave and gives every rank at least two stages.
Plan make_plan(int m, int n, int k) {
    const int nj = m <= 8 ? 1 : (m <= 16 ? 2 : (m <= 32 ? 4 : 8));
    const int m_tiles = cdiv(m, 8 * nj);
    const int stages = cdiv(k, kStageK);
    const int resident = kNumSMs * (nj <= 2 ? 4 : (nj == 4 ? 3 : 1));
    const int wn = cdiv(n, 128) * m_tiles * 8 >= kNumSMs ? 4 : 2;
    const int n_tiles = cdiv(n, 32 * wn);
    const int base = n_tiles * m_tiles;
    int r = 1;
    while (r < 8 && base * r * 2 <= resident && stages / (r * 2) >= 2) r *= 2;
    Plan best{nj, wn, m_tiles, n_tiles, r, cdiv(stages, r)};
    return best;
}

// ---- tensor maps.  cuTensorMapEncodeTiled is a driver entry point; it is looked up
// through the runtime so that the library does not link against libcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult res;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &res) != cudaSuccess ||
            res != cudaDriverEntryPointSuccess)
            ptr = nullptr;
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

// rows x cols row-major matrix of elem_bytes elements with row pitch pitch_bytes; box = box_cols x box_rows
bool make_map(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes, const void* base, uint64_t cols,
              uint64_t rows, uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NJ, bool ZTABLE, int GPS, int WN>
int launch_one(const W4Params& p, const Plan& pl, cudaStream_t st) {
    using L = Layout<NJ, WN, GPS>;
    auto kernel = w4a16_stream_kernel<NJ, ZTABLE, GPS, WN>;
    static bool configured[64] = {};                   // per instantiation and device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LQ2_ERR_CUDA;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
            return LQ2_ERR_CUDA;
        // several CTAs per SM are planned for: ask for the largest shared-memory carve-out
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return LQ2_ERR_CUDA;
        configured[dev] = true;
    }
    alignas(64) CUtensorMap map_w, map_x, map_s, map_z;
    const uint64_t n = uint64_t(p.n), k = uint64_t(p.k), groups = uint64_t(p.k / p.group);
    bool ok = make_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, p.packed, n, k / 8, n * 4, 32, 16, true);
    ok = ok && make_map(&map_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.x, k, uint64_t(p.m), uint64_t(p.ldx) * 2, 64,
                        L::MT, true);
    ok = ok && make_map(&map_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.scales, n, groups, n * 2, L::TN, GPS, false);
    ok = ok && make_map(&map_z, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ZTABLE ? p.zeros : p.scales, n, groups, n * 2,
                        L::TN, GPS, false);
    if (!ok) return LQ2_ERR_CUDA;
    // A grid that needs fewer CTAs per SM than would fit is spread evenly over the SMs by
    // asking for more shared memory than the kernel uses (clusters are otherwise packed densely).
    size_t smem = L::SMEM_BYTES;
    const int per_sm = cdiv(pl.n_tiles * pl.ranks * pl.m_tiles, kNumSMs);
    constexpr int kResident = NJ <= 2 ? 4 : (NJ == 4 ? 3 : 1);
    if (per_sm < kResident && size_t(227 * 1024 / per_sm - 1024) > smem) smem = size_t(227 * 1024 / per_sm - 1024);
    return launch_pdl(kernel, dim3(pl.n_tiles, pl.ranks, pl.m_tiles), dim3(L::THREADS), smem, st, pl.ranks,
                      map_w, map_x, map_s, map_z, p);
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
                        const __half* zeros, __half* y, int m, int n, int k, int group, int silu,
                        void*, size_t, cudaStream_t st) {
    if (m > 8) return LQ2_ERR_SHAPE;
    const Plan pl = make_plan(m, n, k);
    W4Params p;
    p.x = x; p.ldx = ldx; p.packed = packed; p.scales = scales; p.zeros = zeros; p.y = y;
    p.m = m; p.n = n; p.k = k; p.group = group;
    p.stages_per_rank = pl.spr;
    p.early_weights = early_weight_fetch() ? 1 : 0;
    p.silu = silu;
    // Only the 8-row variant is built: larger batches go to the tcgen05 kernel, which is faster
    // from 9 rows on (the kernel template itself is generic in the number of 8-row blocks).
    return launch_z<1>(p, pl, st);
}

}  // namespace lq2
