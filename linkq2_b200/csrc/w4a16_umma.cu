// W4A16 linear for M > 8 (batched decode, verify, prefill): int4 weights are
// dequantised into tensor memory and multiplied on the 5th-generation tensor
// cores (tcgen05.mma) with the accumulator in tensor memory as well.
//
// Replaces the split-K and large-M Triton routes of the reference
// (qslab/kernels/gemlite/triton_kernels/gemm_splitK_A16fWnO16f_int32packing.py:199-412,
//  gemm_A16fWnO16f_int32packing.py:174-373) behind the same buffers.
//
// Shared memory carries only what TMA delivered (about 2 bytes per packed byte); writing
// fp16 weights to it and reading them back for the MMA would need 8 more and make the
// kernel shared-memory-bound well below the HBM rate.
//
// Orientation.  The product is computed transposed, Y^T[n, m] = W[n, :] . X[m, :],
// so that the 128 rows of the MMA are output channels and its N dimension
// (16..128) is the batch: a 32-row decode batch wastes nothing.  Per CTA: 128
// output channels x MB batch rows, K streamed in stages of 128 (64 for batch tiles
// above 64 rows).
//
// Warp roles (10 warps):
//   warp 0      producer: tiled TMA loads of the stage's packed words [k/8 x 128]
//               int32, its activation tile as [MB x 64] fp16 boxes (128-byte swizzle,
//               K-major: already the MMA's B operand layout), scales and zero points
//   warps 2-9   dequantise: thread (n, half) turns 4 packed words of channel n into
//               4 x 8 fp16 values, (u - z) * s rounded once exactly as the reference
//               (triton_kernels/utils.py:66-71; integer-valued zero points), and
//               stores them with tcgen05.st into the A tile in tensor memory (lane =
//               channel, 32-bit column = two consecutive k): the 4x expanded
//               weights never pass through shared memory
//   warp 1      issues tcgen05.mma (M=128, N=MB, K=16, A from TMEM, B from shared
//               memory, fp32 accumulate in TMEM) and commits each stage to the
//               mbarriers that free its buffers
//   warps 2-5   epilogue: tcgen05.ld of the accumulator, then the same cluster
//               split-K reduction through distributed shared memory as the
//               streaming kernel, fp16 store
// All waits are bounded (see mbar_wait_bounded).
#include <cooperative_groups.h>
#include <cuda.h>
#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace lq2 {

namespace {

constexpr int kMaxSmemPerCta = 227 * 1024;
constexpr int kUM = 128;          // output channels per CTA (MMA M)
// k per pipeline stage: 128 for batch tiles up to 64 rows (half as many barrier rounds per
// byte as 64, measured 8-15 % faster), 64 beyond, where the activation tile of a stage grows
__host__ __device__ constexpr int stage_k(int mb) { return mb <= 64 ? 128 : 64; }
constexpr int kUThreads = 320;    // 10 warps: TMA producer, MMA issuer, 8 dequantisers (+ one more issuer, see ISS)
constexpr int kIssuer2 = 10;      // warp index of the second issuer
constexpr int kDequantThreads = 256;

struct UParams {
    __half* y;
    int m, n, k, group;
    int stages_per_rank;
    int early_weights;    // request weight bytes before the previous kernel of the stream has finished
    int silu;             // columns are interleaved [4 gate | 4 up]: write silu(gate) * up, N / 2 wide
    PushTarget push;      // tensor-parallel peers that receive the output as flagged words (world 0: none)
    const unsigned int* exchange_calls;   // this rank's exchange call counter (null without peers)
};

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
// Number of waits that gave up; stays 0 in a healthy run.
__device__ unsigned int g_lq2_umma_wait_timeouts = 0;
constexpr int kMaxWaitPolls = 1 << 22;
// Bounded wait: after kMaxWaitPolls unsuccessful polls the wait is abandoned and counted,
// and the kernel runs on to its end (wrong output, but no spinning GPU).
__device__ __forceinline__ void mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < kMaxWaitPolls; ++i)
        if (mbar_try_wait(bar, parity)) return;
    atomicAdd(&g_lq2_umma_wait_timeouts, 1u);
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];\n" ::"l"(map) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n"
        ::"r"(dst), "l"(map), "r"(c0), "r"(c1), "r"(bar) : "memory");
}

// ---- cluster barrier, split into its two halves
__device__ __forceinline__ void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory"); }

// ---- tcgen05 wrappers (cta_group::1)
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_dst), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// arrive on an mbarrier once all MMAs issued so far by this thread have completed
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]: the A operand (M = 128 lanes x K/2 columns, two fp16 per 32-bit
// column, lower k in the lower half) is read from tensor memory
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n.reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// store 16 consecutive 32-bit columns of this thread's TMEM lane (completion: tcgen05.wait::st)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]) : "memory");
}
// 16 consecutive accumulator columns of this thread's TMEM lane from each of two accumulators, summed
// (one wait for both loads)
__device__ __forceinline__ void tmem_ld16_sum2(uint32_t taddr_a, uint32_t taddr_b, float (&v)[16]) {
    uint32_t r[16], q[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr_a) : "memory");
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]), "=r"(q[6]), "=r"(q[7]),
          "=r"(q[8]), "=r"(q[9]), "=r"(q[10]), "=r"(q[11]), "=r"(q[12]), "=r"(q[13]), "=r"(q[14]), "=r"(q[15])
        : "r"(taddr_b) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]) + __uint_as_float(q[i]);
}
// 16 consecutive accumulator columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of 64 fp16 (128 B),
// 8-row groups 1024 B apart.  Fields: start address >> 4 in bits [0,14), leading-dimension
// byte offset >> 4 in [16,30) (unused by swizzled K-major layouts), stride-dimension byte
// offset >> 4 in [32,46), descriptor version 1 in [46,48), layout type SWIZZLE_128B = 2 in [61,64).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator (bit 4), fp16 A and B (formats 0),
// both K-major, N >> 3 in bits [17,23), M >> 4 in bits [24,29).
__host__ __device__ constexpr uint32_t umma_idesc(int mma_m, int mma_n) {
    return (1u << 4) | (uint32_t(mma_n >> 3) << 17) | (uint32_t(mma_m >> 4) << 24);
}

// Two rings: one in shared memory for what TMA delivers (packed words, activations, scales:
// ~9 KB per stage at MB = 32), which sets the bytes in flight, and one in tensor memory for
// the dequantised A tiles (32 columns each), so the 4x expanded weights never touch shared
// memory.
template <int MB, int GPSU>
struct ULayout {
    static constexpr int UK = stage_k(MB);
    // A tiles in tensor memory.  A 128-k tile takes 64 columns; one of them plus the two accumulators
    // of a 32-row batch fits a 128-column allocation, so three CTAs share an SM.  (Two A tiles with two
    // CTAs per SM were measured and are no faster: 2.8 against 2.6 stages per microsecond and SM.)
    static constexpr int A_STAGES = UK == 128 ? 1 : 3;
    static constexpr int A_COLS = UK / 2;                           // 32-bit TMEM columns per A tile (two fp16 each)
    static constexpr int XBOX_BYTES = (MB * 128 + 1023) / 1024 * 1024;   // [MB m][64 k] fp16, swizzled
    static constexpr int X_BYTES = (UK / 64) * XBOX_BYTES;
    static constexpr int RAW_BYTES = (UK / 8) * kUM * 4;            // [UK/8 k8][128 n] int32
    static constexpr int S_BYTES = GPSU * kUM * 2;                  // [GPSU][128 n] fp16
    static constexpr int RAW_OFF = X_BYTES, S_OFF = RAW_OFF + RAW_BYTES, Z_OFF = S_OFF + S_BYTES;
    static constexpr int R_STAGE_BYTES = (Z_OFF + S_BYTES + 1023) / 1024 * 1024;   // x tile first: 1 KiB aligned
    static constexpr int R_STAGES = UK == 128 ? (MB <= 16 ? 4 : 3) : (MB <= 64 ? 6 : (MB <= 128 ? 4 : 3));
    static constexpr int TX_BYTES = (UK / 64) * MB * 128 + RAW_BYTES;   // + S_BYTES (x2 with zero points)
    static constexpr int R_RING_OFF = 0;
    static constexpr int RING_BYTES = R_RING_OFF + R_STAGES * R_STAGE_BYTES;
    static constexpr int RED_BYTES = MB * kUM * 4;
    // Split-K reduction.  Up to 64 batch rows every CTA has a receive area of its own
    // ([source rank][MB][128 / ranks] fp32, never aliased with the ring) into which the
    // ranks of its cluster push their partial sums; beyond, the partial tile is staged
    // in the idle ring and pulled by the owners of the column slices.
    static constexpr bool PUSH = MB <= 64;
    static constexpr int RECV_OFF = RING_BYTES;
    static constexpr int DATA_BYTES = PUSH ? RING_BYTES + RED_BYTES : (RING_BYTES > RED_BYTES ? RING_BYTES : RED_BYTES);
    static constexpr int NBARS = 2 * R_STAGES + (1 + (UK == 128 ? 2 : 1)) * A_STAGES + 1;
    static constexpr int SMEM_BYTES = 1024 + DATA_BYTES + NBARS * 8 + 16;
    static constexpr int ACC_COLS = MB < 32 ? 32 : MB;
    // One thread issues a tcgen05.mma of this size about every 115 cycles, whatever the tensor pipe is
    // doing, and with a single A tile the stage's MMAs sit between "tile written" and "tile free" on the
    // CTA's critical path.  With 128-k stages two warps therefore issue half of a stage's MMAs each, into
    // accumulators of their own (their rates add up); the epilogue sums the two.
    static constexpr int ISS = UK == 128 ? 2 : 1;
    static constexpr int THREADS = kUThreads + 32 * (ISS - 1);
    static constexpr int TMEM_NEED = ISS * ACC_COLS + A_STAGES * A_COLS;
    static constexpr int TMEM_COLS = TMEM_NEED <= 64 ? 64 : (TMEM_NEED <= 128 ? 128 : (TMEM_NEED <= 256 ? 256 : 512));
    static_assert(TMEM_NEED <= 512, "tensor memory has 512 columns");
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory per CTA");
};


// CTAs per SM the plan counts on (shared memory and tensor-memory columns allow them; the
// launch bounds make the register allocation follow)
__host__ __device__ constexpr int resident_ctas(int mb) { return mb <= 32 ? 3 : (mb <= 128 ? 2 : 1); }

template <int MB, bool ZTABLE, int GPSU>
__global__ void __launch_bounds__((ULayout<MB, GPSU>::THREADS), resident_ctas(MB))
w4a16_umma_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                  const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                  const UParams p) {
    using L = ULayout<MB, GPSU>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int RS = L::R_STAGES, AS = L::A_STAGES, UK = L::UK, ISS = L::ISS;
    const uint32_t bars = smem_u32(smem + L::DATA_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::DATA_BYTES + L::NBARS * 8);
    volatile unsigned int* push_seq = tmem_slot + 2;          // the 16 bytes behind the barriers hold both
    auto raw_full = [&](int s) { return bars + 8 * s; };               // TMA bytes of raw stage s landed
    auto raw_free = [&](int s) { return bars + 8 * (RS + s); };        // MMAs that read its activations are done
    // k-half h of A tile s written by the dequant warps that own it (all of them when there is one issuer)
    auto a_full = [&](int s, int h) { return bars + 8 * (2 * RS + ISS * s + h); };
    auto a_free = [&](int s) { return bars + 8 * (2 * RS + ISS * AS + s); };   // MMAs that read A tile s are done
    const uint32_t acc_full = bars + 8 * (2 * RS + (ISS + 1) * AS);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile_n0 = blockIdx.x * kUM;
    if (threadIdx.x == 0) {                  // the tensor maps' descriptors are on their way before the first copy needs them
        prefetch_tensormap(&map_w);
        prefetch_tensormap(&map_x);
        prefetch_tensormap(&map_s);
        prefetch_tensormap(&map_z);
    }
    const int m0 = blockIdx.z * MB;
    const int rows = min(MB, p.m - m0);
    const int total_stages = (p.k + UK - 1) / UK;
    const int ranks = gridDim.y, rank = blockIdx.y;
    const int s0 = min(total_stages, rank * p.stages_per_rank);
    const int s1 = min(total_stages, s0 + p.stages_per_rank);
    const int my_stages = s1 - s0;

    if (tid == 0) {
        for (int i = 0; i < RS; ++i) {
            mbar_init(raw_full(i), 1);
            mbar_init(raw_free(i), ISS);
        }
        for (int i = 0; i < AS; ++i) {
            for (int h = 0; h < ISS; ++h) mbar_init(a_full(i, h), kDequantThreads / 32 / ISS);
            mbar_init(a_free(i), ISS);
        }
        mbar_init(acc_full, ISS);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), L::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Only now may the next kernel of the stream be scheduled next to this CTA: had it been let in
    // before the allocation above, its CTAs could take the tensor memory this one still needs and then
    // wait for this grid to finish.
    pdl_launch_dependents();
    // first half of a cluster barrier: by the time the epilogue waits for it, every CTA of
    // the cluster is known to be running, which remote shared-memory stores require
    if (L::PUSH && ranks > 1) cluster_arrive_release();
    const uint32_t tmem_base = *tmem_slot;
    unsigned char* r_ring = smem + L::R_RING_OFF;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        auto load_weights = [&](int it) {
            const int slot = it % RS, s = s0 + it;
            const uint32_t base = smem_u32(r_ring + slot * L::R_STAGE_BYTES);
            mbar_arrive_expect_tx(raw_full(slot), L::TX_BYTES + L::S_BYTES * (ZTABLE ? 2 : 1));
            tma_load_2d(base + L::RAW_OFF, &map_w, tile_n0, s * (UK / 8), raw_full(slot));
            const int gi = (GPSU == 1) ? (s * UK) / p.group : s * GPSU;
            tma_load_2d(base + L::S_OFF, &map_s, tile_n0, gi, raw_full(slot));
            if (ZTABLE) tma_load_2d(base + L::Z_OFF, &map_z, tile_n0, gi, raw_full(slot));
        };
        auto load_activations = [&](int it) {
            const int slot = it % RS, s = s0 + it;
            const uint32_t base = smem_u32(r_ring + slot * L::R_STAGE_BYTES);
#pragma unroll
            for (int b = 0; b < UK / 64; ++b)
                tma_load_2d(base + b * L::XBOX_BYTES, &map_x, s * UK + 64 * b, m0, raw_full(slot));
        };
        // When the caller has declared the weights constant, the first ring of weight bytes
        // is requested before the previous kernel of the stream has finished; the
        // activations, which that kernel may still be writing, only after pdl_wait().
        const int ahead = min(my_stages, RS);
        if (!p.early_weights) pdl_wait();
        if (lane == 0)
            for (int it = 0; it < ahead; ++it) load_weights(it);
        if (p.early_weights) pdl_wait();
        if (lane == 0)
            for (int it = 0; it < ahead; ++it) load_activations(it);
        __syncwarp();
        for (int it = ahead; it < my_stages; ++it) {
            mbar_wait_bounded(raw_free(it % RS), ((it / RS) - 1) & 1);
            if (lane == 0) {
                load_weights(it);
                load_activations(it);
            }
            __syncwarp();
        }
    } else if (warp == 1 || (ISS == 2 && warp == kIssuer2)) {
        // ------------------------------------------------------------ MMA issuer(s)
        pdl_wait();
        const int half = warp == 1 ? 0 : 1;                   // which k-half of every stage, and which accumulator
        constexpr int KSTEPS = UK / 16 / ISS;
        constexpr uint32_t idesc = umma_idesc(kUM, MB);
        constexpr int U = RS % AS == 0 && UK == 128 ? RS : 1;   // unrolled over the raw ring, as the dequantisers are
        for (int it0 = 0; it0 < my_stages; it0 += U) {
#pragma unroll
          for (int us = 0; us < U; ++us) {
            const int it = it0 + us;
            if (it >= my_stages) break;
            const int rslot = U == 1 ? it % RS : us, aslot = U == 1 ? it % AS : us % AS;
            mbar_wait_bounded(a_full(aslot, half), (it / AS) & 1);
            tc_fence_after();
            if (lane == 0) {
                const uint32_t a_tmem = tmem_base + ISS * L::ACC_COLS + aslot * L::A_COLS;
                const uint32_t xbase = smem_u32(r_ring + rslot * L::R_STAGE_BYTES);
#pragma unroll
                for (int ks = 0; ks < KSTEPS; ++ks) {
                    // a K step of 16 fp16: 8 TMEM columns of A, 32 bytes inside the swizzled rows of B
                    // (a 64-k box holds four such steps)
                    const int kk = half * KSTEPS + ks;
                    umma_f16_ts(tmem_base + half * L::ACC_COLS, a_tmem + kk * 8,
                                smem_desc_sw128(xbase + (kk >> 2) * L::XBOX_BYTES + (kk & 3) * 32), idesc,
                                (it > 0 || ks > 0) ? 1u : 0u);
                }
                umma_commit(a_free(aslot));                   // both buffers are reusable once these MMAs are done
                umma_commit(raw_free(rslot));
                if (it == my_stages - 1) umma_commit(acc_full);
            }
            __syncwarp();
          }
        }
    } else if (warp < 2 + kDequantThreads / 32) {
        // ------------------------------------------------------------ dequantise
        pdl_wait();
        // The exchange's call counter is read here, long before the epilogue needs it, so that its memory
        // round trip is off the end of the kernel; the kernels that advance it precede this one in the stream.
        if (p.exchange_calls && tid == 64)
            *push_seq = *reinterpret_cast<const volatile unsigned int*>(p.exchange_calls) + 1;   // calls completed + 1
        // A warp reaches the 32 TMEM lanes of its quarter (warp % 4); lane = output channel.  Two
        // warps share a quarter and take k8 rows 0-3 and 4-7 of the stage.
        const int quarter = warp & 3, khalf = (warp - 2) >> 2;
        const int nl = quarter * 32 + lane;
        const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
        const __half2 k1024 = __floats2half2_rn(1024.f, 1024.f);
        const __half2 k64 = __floats2half2_rn(64.f, 64.f);
        constexpr int W = UK / 16;                            // packed words per thread per stage
        // The stores of a stage are left in flight while the next stage's words are fetched
        // from shared memory; only then are they waited for and the tile handed to the MMA warp.
        auto publish = [&](int it_done) {
            asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(a_full(it_done % AS, ISS == 2 ? khalf : 0));
        };
        // With a single A tile the loop is unrolled over the raw ring, which makes the stage
        // slot, its shared-memory addresses and its barrier compile-time constants.
        constexpr int U = RS % AS == 0 && UK == 128 ? RS : 1;
        uint32_t ring_phase = 0;                              // (it / RS) & 1 when U == RS
        for (int it0 = 0; it0 < my_stages; it0 += U, ring_phase ^= 1u) {
#pragma unroll
          for (int us = 0; us < U; ++us) {
            const int it = it0 + us;
            if (it >= my_stages) break;
            const int rslot = U == 1 ? it % RS : us, aslot = U == 1 ? it % AS : us % AS;
            const unsigned char* rbase = r_ring + rslot * L::R_STAGE_BYTES;
            mbar_wait_bounded(raw_full(rslot), U == 1 ? uint32_t(it / RS) & 1u : ring_phase);
            const uint32_t* raw = reinterpret_cast<const uint32_t*>(rbase + L::RAW_OFF);
            const __half* sc = reinterpret_cast<const __half*>(rbase + L::S_OFF);
            const __half* zc = reinterpret_cast<const __half*>(rbase + L::Z_OFF);
            uint32_t wv[W];
#pragma unroll
            for (int r = 0; r < W; ++r) wv[r] = raw[(W * khalf + r) * kUM + nl];   // k = 8 * row .. + 7 of channel nl
            // quantization group of each block of four words (32 k); a thread covers UK/2 consecutive k
            __half sraw[W / 4], zraw[W / 4];
#pragma unroll
            for (int b = 0; b < W / 4; ++b) {
                const int gq = ((W * khalf + 4 * b) * 8 * GPSU) / UK;
                sraw[b] = sc[gq * kUM + nl];
                zraw[b] = ZTABLE ? zc[gq * kUM + nl] : __float2half_rn(8.f);
            }
            if (it > 0) publish(it - 1);
            if (it >= AS) {
                mbar_wait_bounded(a_free(aslot), ((it / AS) - 1) & 1);
                tc_fence_after();
            }
#pragma unroll
            for (int b = 0; b < W / 4; ++b) {
                const __half2 s2 = __half2half2(sraw[b]);
                const __half2 z2 = __half2half2(zraw[b]);
                const __half2 zlo = __hadd2(z2, k1024), zhi = __hneg2(__hadd2(z2, k64));
                uint32_t cols[16];
#pragma unroll
                for (int r4 = 0; r4 < 4; ++r4) {
                    const uint32_t w = wv[4 * b + r4];
                    const uint32_t w8 = w >> 8;
                    // (u - z) * s rounded once; the masks give the pairs (0,4) (1,5) (2,6) (3,7)
                    const uint32_t v04 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(and_or(w, 0x000f000fu, 0x64006400u)), zlo), s2));
                    const uint32_t v15 = h2_as_u32(__hmul2(__hfma2(u32_as_h2(and_or(w, 0x00f000f0u, 0x64006400u)), k16th, zhi), s2));
                    const uint32_t v26 = h2_as_u32(__hmul2(__hsub2(u32_as_h2(and_or(w8, 0x000f000fu, 0x64006400u)), zlo), s2));
                    const uint32_t v37 = h2_as_u32(__hmul2(__hfma2(u32_as_h2(and_or(w8, 0x00f000f0u, 0x64006400u)), k16th, zhi), s2));
                    cols[4 * r4 + 0] = __byte_perm(v04, v15, 0x5410);        // k0 k1
                    cols[4 * r4 + 1] = __byte_perm(v26, v37, 0x5410);        // k2 k3
                    cols[4 * r4 + 2] = __byte_perm(v04, v15, 0x7632);        // k4 k5
                    cols[4 * r4 + 3] = __byte_perm(v26, v37, 0x7632);        // k6 k7
                }
                tmem_st16(tmem_base + (uint32_t(quarter * 32) << 16) + ISS * L::ACC_COLS + aslot * L::A_COLS +
                              khalf * (UK / 4) + 16 * b, cols);
            }
          }
        }
        if (my_stages > 0) publish(my_stages - 1);
    }

    // ---- epilogue: warps 2-5 read the accumulator (TMEM lane = output channel)
    cg::cluster_group cluster = cg::this_cluster();
    if (warp >= 2 && warp < 6) {
        if (my_stages > 0) {
            mbar_wait_bounded(acc_full, 0);
            tc_fence_after();
        }
    }
    if constexpr (L::PUSH) {
        // Push: rank q of the cluster owns channels [q * W, (q + 1) * W) of the tile.  Every rank
        // writes its partial sums for those channels straight from registers into q's receive
        // area (remote shared memory), one cluster barrier follows, and q adds the ranks' parts
        // in rank order.  Nobody reads remote memory after the barrier, so a CTA may leave as
        // soon as it has written its slice.
        const int W = kUM / ranks;
        float* recv = reinterpret_cast<float*>(smem + L::RECV_OFF);   // [ranks][MB][W]
        if (ranks > 1) cluster_wait_acquire();                        // all CTAs of the cluster are running
        if (warp >= 2 && warp < 6) {
            const int quarter = warp & 3;                  // TMEM lanes 32*quarter .. +31 belong to this warp
            const int nl = quarter * 32 + lane;
            const int dest = nl / W, c = nl - dest * W;
            float* dst = (ranks > 1 ? cluster.map_shared_rank(recv, dest) : recv) + size_t(rank) * MB * W + c;
#pragma unroll 1
            for (int c0 = 0; c0 < MB; c0 += 16) {
                float v[16];
                if (my_stages > 0) {
                    const uint32_t acc = tmem_base + (uint32_t(quarter * 32) << 16) + c0;
                    if (ISS == 2) tmem_ld16_sum2(acc, acc + L::ACC_COLS, v); else tmem_ld16(acc, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) dst[(c0 + i) * W] = v[i];
            }
        }
        tc_fence_before();
        __syncthreads();
        if (warp == 1) tmem_dealloc(tmem_base, L::TMEM_COLS);
        if (ranks > 1) {
            cluster_arrive_release();
            cluster_wait_acquire();
        }
        auto slice_sum = [&](int ml, int col) {
            float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int q = 0; q < ranks; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(recv + (size_t(q) * MB + ml) * W + col);
                sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
            }
            return sum;
        };
        if (p.silu) {
            const int octs = W / 8;                        // [4 gate | 4 up] blocks of my slice
            for (int e = tid; e < rows * octs; e += L::THREADS) {
                const int ml = e / octs, col = (e - ml * octs) * 8;
                const int nn = tile_n0 + rank * W + col;
                if (nn < p.n)
                    *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * (p.n / 2) + nn / 2) =
                        silu_mul_quad(slice_sum(ml, col), slice_sum(ml, col + 4));
            }
        } else {
            // Row-split projections under tensor parallelism: besides y, every finished quad goes
            // straight into the peers' exchange buffers as one flagged 16-byte word {2 halves, seq,
            // 2 halves, seq} (the format lq2_rmsnorm_allreduce gathers), so the transfer overlaps
            // the rest of this kernel instead of starting when the consumer does.
            const int world = p.push.world, me = p.push.rank;
            unsigned int seq = 0;
            size_t ll = 0;
            if (world > 1) {
                seq = *push_seq;                       // written before the barrier above
                ll = llslots_offset(world, p.push.max_bytes) +
                     (size_t(seq & 1u) * world + me) * 2 * p.push.max_bytes;
            }
            const int quads = W / 4;
            for (int e = tid; e < rows * quads; e += L::THREADS) {
                const int ml = e / quads, col = (e - ml * quads) * 4;
                const float4 sum = slice_sum(ml, col);
                const int nn = tile_n0 + rank * W + col;
                if (nn < p.n) {
                    const uint32_t lo = h2_as_u32(__floats2half2_rn(sum.x, sum.y));
                    const uint32_t hi = h2_as_u32(__floats2half2_rn(sum.z, sum.w));
                    *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * p.n + nn) = make_uint2(lo, hi);
                    if (world > 1) {
                        const size_t off = ll + (size_t(m0 + ml) * (p.n / 8) + (nn >> 3)) * 32 + ((nn >> 2) & 1) * 16;
                        const uint4 word = make_uint4(lo, seq, hi, seq);
#pragma unroll
                        for (int peer = 0; peer < kMaxWorld; ++peer)   // constant indices: the table stays in parameter space
                            if (peer < world && peer != me) *reinterpret_cast<uint4*>(p.push.peers.base[peer] + off) = word;
                    }
                }
            }
        }
    } else {
        float* red = reinterpret_cast<float*>(smem);          // [MB][128], in the idle ring
        __syncthreads();                                       // the ring is idle from here on
        if (warp >= 2 && warp < 6) {
            const int quarter = warp & 3;
            const int nl = quarter * 32 + lane;
#pragma unroll
            for (int c0 = 0; c0 < MB; c0 += 16) {
                float v[16];
                if (my_stages > 0) {
                    const uint32_t acc = tmem_base + (uint32_t(quarter * 32) << 16) + c0;
                    if (ISS == 2) tmem_ld16_sum2(acc, acc + L::ACC_COLS, v); else tmem_ld16(acc, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) v[i] = 0.f;
                }
#pragma unroll
                for (int i = 0; i < 16; ++i) red[(c0 + i) * kUM + nl] = v[i];
            }
        }
        tc_fence_before();
        __syncthreads();
        if (warp == 1) tmem_dealloc(tmem_base, L::TMEM_COLS);
        if (ranks > 1) cluster.sync();
        {
            constexpr int QUADS = kUM / 4;
            const int q0 = rank * QUADS / ranks, q1 = (rank + 1) * QUADS / ranks;
            const int quads = q1 - q0;
            auto tile_sum = [&](int ml, int col) {
                float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int q = 0; q < ranks; ++q) {
                    const float* src = ranks > 1 ? cluster.map_shared_rank(red, q) : red;
                    const float4 v = *reinterpret_cast<const float4*>(src + ml * kUM + col);
                    sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
                }
                return sum;
            };
            if (p.silu) {                                  // q0 is even for every power-of-two cluster size
                const int octs = quads / 2;
                for (int e = tid; e < rows * octs; e += L::THREADS) {
                    const int ml = e / octs, col = (q0 + 2 * (e % octs)) * 4;
                    const int nn = tile_n0 + col;
                    if (nn < p.n)
                        *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * (p.n / 2) + nn / 2) =
                            silu_mul_quad(tile_sum(ml, col), tile_sum(ml, col + 4));
                }
            } else {
                for (int e = tid; e < rows * quads; e += L::THREADS) {
                    const int ml = e / quads, col = (q0 + e % quads) * 4;
                    const float4 sum = tile_sum(ml, col);
                    const int nn = tile_n0 + col;
                    if (nn < p.n) {
                        const __half2 lo = __floats2half2_rn(sum.x, sum.y);
                        const __half2 hi = __floats2half2_rn(sum.z, sum.w);
                        *reinterpret_cast<uint2*>(p.y + int64_t(m0 + ml) * p.n + nn) = make_uint2(h2_as_u32(lo), h2_as_u32(hi));
                    }
                }
            }
        }
        if (ranks > 1) cluster.sync();                                 // nobody leaves while its tile is still being read
    }
}

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

bool make_map(CUtensorMap* map, CUtensorMapDataType type, const void* base, uint64_t cols, uint64_t rows,
              uint64_t pitch_bytes, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct UPlan {
    int mb, m_tiles, n_tiles, ranks, spr;
};

// Batch tile and cluster size from shapes only: the largest power-of-two K split that
// keeps the grid within one resident wave and leaves every rank at least four stages.
UPlan make_uplan(int m, int n, int k) {
    UPlan p;
    // 128-row batch tiles at two CTAs per SM beat 256-row tiles at one at every M measured
    // (gate_up geometry: 126 vs 159 us at M = 512, 439 vs 522 us at M = 2048)
    p.mb = m <= 16 ? 16 : (m <= 32 ? 32 : (m <= 64 ? 64 : 128));
    p.m_tiles = cdiv(m, p.mb);
    p.n_tiles = cdiv(n, kUM);
    const int stages = cdiv(k, stage_k(p.mb));
    const int base = p.n_tiles * p.m_tiles;
    int r = 1;
    const int resident = kNumSMs * resident_ctas(p.mb);
    while (r < 8 && base * r * 2 <= resident && stages / (r * 2) >= 4) r *= 2;
    p.ranks = r;
    p.spr = cdiv(stages, r);
    return p;
}

template <int MB, bool ZTABLE, int GPSU>
int launch_umma(const __half* x, int64_t ldx, const int32_t* packed, const __half* scales, const __half* zeros,
                const UParams& p, const UPlan& pl, cudaStream_t st) {
    using L = ULayout<MB, GPSU>;
    auto kernel = w4a16_umma_kernel<MB, ZTABLE, GPSU>;
    static bool configured[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LQ2_ERR_CUDA;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemPerCta) != cudaSuccess)
            return LQ2_ERR_CUDA;
        // several CTAs per SM are planned for: ask for the largest shared-memory carve-out
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared) != cudaSuccess)
            return LQ2_ERR_CUDA;
        configured[dev] = true;
    }
    alignas(64) CUtensorMap map_w, map_x, map_s, map_z;
    const uint64_t n = uint64_t(p.n), k = uint64_t(p.k), groups = uint64_t(p.k / p.group);
    bool ok = make_map(&map_w, CU_TENSOR_MAP_DATA_TYPE_INT32, packed, n, k / 8, n * 4, kUM, L::UK / 8, false);
    ok = ok && make_map(&map_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x, k, uint64_t(p.m), uint64_t(ldx) * 2, 64, MB, true);
    ok = ok && make_map(&map_s, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, scales, n, groups, n * 2, kUM, GPSU, false);
    ok = ok && make_map(&map_z, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ZTABLE ? zeros : scales, n, groups, n * 2, kUM, GPSU, false);
    if (!ok) return LQ2_ERR_CUDA;
    // A grid that needs fewer CTAs per SM than would fit is spread evenly by asking for more
    // shared memory than the kernel uses: 256 CTAs land two per SM on 108 SMs and one on 40
    // instead of three on some and none on others (clusters are otherwise packed densely).
    size_t smem = L::SMEM_BYTES;
    const int ctas = pl.n_tiles * pl.ranks * pl.m_tiles;
    const int per_sm = cdiv(ctas, kNumSMs);
    if (per_sm < resident_ctas(MB)) smem = std::max(smem, size_t(kMaxSmemPerCta / per_sm - 1024));
    return launch_pdl(kernel, dim3(pl.n_tiles, pl.ranks, pl.m_tiles), dim3(L::THREADS), smem, st, pl.ranks,
                      map_w, map_x, map_s, map_z, p);
}

template <int MB, bool ZTABLE>
int launch_umma_g(const __half* x, int64_t ldx, const int32_t* packed, const __half* scales, const __half* zeros,
                  const UParams& p, const UPlan& pl, cudaStream_t st) {
    constexpr int UK = stage_k(MB);                    // groups per stage: 1, 2 or 4
    if (p.group >= UK) return launch_umma<MB, ZTABLE, 1>(x, ldx, packed, scales, zeros, p, pl, st);
    if (p.group * 2 == UK) return launch_umma<MB, ZTABLE, 2>(x, ldx, packed, scales, zeros, p, pl, st);
    if constexpr (UK == 128) return launch_umma<MB, ZTABLE, 4>(x, ldx, packed, scales, zeros, p, pl, st);
    return LQ2_ERR_SHAPE;
}

template <int MB>
int launch_umma_z(const __half* x, int64_t ldx, const int32_t* packed, const __half* scales, const __half* zeros,
                  const UParams& p, const UPlan& pl, cudaStream_t st) {
    return zeros ? launch_umma_g<MB, true>(x, ldx, packed, scales, zeros, p, pl, st)
                 : launch_umma_g<MB, false>(x, ldx, packed, scales, zeros, p, pl, st);
}

}  // namespace

int w4a16_umma_launch(const __half* x, int64_t ldx, const int32_t* packed, const __half* scales,
                      const __half* zeros, __half* y, int m, int n, int k, int group, int silu,
                      const PushTarget* push, cudaStream_t st) {
    const UPlan pl = make_uplan(m, n, k);
    if (pl.m_tiles > 65535) return LQ2_ERR_SHAPE;
    UParams p;
    p.y = y; p.m = m; p.n = n; p.k = k; p.group = group; p.stages_per_rank = pl.spr;
    p.early_weights = early_weight_fetch() ? 1 : 0;
    p.silu = silu;
    p.push = PushTarget{};
    p.exchange_calls = nullptr;
    if (push) {
        if (pl.mb > 64 || silu) return LQ2_ERR_SHAPE;      // only the pushed-reduction epilogue carries it
        p.push = *push;
        p.exchange_calls = reinterpret_cast<const unsigned int*>(push->peers.base[push->rank]);
    }
    switch (pl.mb) {
        case 16: return launch_umma_z<16>(x, ldx, packed, scales, zeros, p, pl, st);
        case 32: return launch_umma_z<32>(x, ldx, packed, scales, zeros, p, pl, st);
        case 64: return launch_umma_z<64>(x, ldx, packed, scales, zeros, p, pl, st);
        default: return launch_umma_z<128>(x, ldx, packed, scales, zeros, p, pl, st);
    }
}

}  // namespace lq2
