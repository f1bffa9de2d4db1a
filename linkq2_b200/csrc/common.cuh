// Shared device helpers for the sm_100a kernels of this library.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/linkq2_b200.h"

namespace lq2 {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline int check_launch() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LQ2_OK : LQ2_ERR_CUDA;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- Programmatic dependent launch.  Every kernel of this library is launched with the
// "programmatic stream serialization" attribute and follows one protocol:
//   * pdl_launch_dependents() as early as possible, but after any tensor-memory
//     allocation (a dependent CTA that got the columns first would wait for this grid
//     while this grid waits for the columns): once all CTAs of the grid have passed it,
//     the next kernel of the stream may be scheduled onto free SM resources, so its
//     launch latency and prologue overlap this grid's tail;
//   * pdl_wait() before the first access to memory that an earlier kernel may have
//     written, and before the first write to memory an earlier kernel may still read.
//     It returns when all earlier grids have completed and their writes are visible.
// Since every kernel waits before it completes, completion stays transitive along the
// stream.  Kernels that are not launched with the attribute see both as no-ops.
// The only accesses ever issued before pdl_wait() are loads of quantized weights and
// their scales/zero points, and only after the caller has declared them constant
// (lq2_w4a16_set_constant_weights; early_weight_fetch() below reads that switch).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

bool early_weight_fetch();   // defined next to the extern "C" switch
bool pdl_enabled();          // false when the environment has LQ2_DISABLE_PDL=1 (diagnostic: plain stream order)

// Launch `kernel` with the programmatic-serialization attribute (and, when cluster_y > 1,
// as thread-block clusters of (1, cluster_y, 1)).
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      int cluster_y, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl_enabled()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster_y > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = cluster_y;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kernel, KArgs(args)...) == cudaSuccess ? LQ2_OK : LQ2_ERR_CUDA;
}

// ---- layout of a rank's tensor-parallel exchange buffer (described in tp_allreduce.cu)
constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 256;
struct PeerTable {
    unsigned char* base[kMaxWorld];
};
// peers.base[i] for a run-time i without indexing the by-value table dynamically (which
// would make the compiler copy it to local memory at kernel entry)
__device__ __forceinline__ unsigned char* peer_base(const PeerTable peers, int i) {
    unsigned char* p = nullptr;
#pragma unroll
    for (int k = 0; k < kMaxWorld; ++k)
        if (k == i) p = peers.base[k];
    return p;
}
// Where a projection kernel pushes its output for the all-reduce that follows it; world == 0: nowhere.
struct PushTarget {
    PeerTable peers;
    int rank, world;
    size_t max_bytes;
};
__host__ __device__ inline size_t flags_offset() { return 256; }
__host__ __device__ inline size_t slots_offset(int world) {
    const size_t raw = flags_offset() + size_t(2) * world * kMaxCtas * 4;
    return (raw + 255) / 256 * 256;
}
__host__ __device__ inline size_t llslots_offset(int world, size_t max_bytes) {
    return slots_offset(world) + size_t(2) * world * max_bytes;
}

// ---- warp-level tensor core op used as a dot-product engine by the
// ---- bandwidth-bound kernels: D(16x8,f32) += A(16x16,f16) * B(16x8,f16)
__device__ __forceinline__ void mma_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with a zero C operand: D = A * B (starts a fresh accumulator without clearing registers)
__device__ __forceinline__ void mma_m16n8k16_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                  uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// (a & b) | c in one LOP3
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// fp16(silu(fp32(g))) * u on a pair of fp16 values: F.silu(gate) * up of Qwen3MLP.forward
// (qslab/runtime/model/qwen3.py:64) with torch's rounding points.
__device__ __forceinline__ __half2 silu_mul2(__half2 g, __half2 u) {
    const float2 a = __half22float2(g);
    const __half2 s = __floats2half2_rn(a.x / (1.0f + expf(-a.x)), a.y / (1.0f + expf(-a.y)));
    return __hmul2(s, u);
}
// The same applied to the fp32 sums of four gate and four up channels (rounded to fp16 first,
// as the unfused projection would have stored them).
__device__ __forceinline__ uint2 silu_mul_quad(const float4& g, const float4& u) {
    const __half2 lo = silu_mul2(__floats2half2_rn(g.x, g.y), __floats2half2_rn(u.x, u.y));
    const __half2 hi = silu_mul2(__floats2half2_rn(g.z, g.w), __floats2half2_rn(u.z, u.w));
    return make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
}

// Streaming 128-bit / 64-bit global loads: the data is read once, keep it out of L1.
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n"
                 : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}
__device__ __forceinline__ uint32_t ldg_stream_u1(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];\n" : "=r"(v) : "l"(p));
    return v;
}

}  // namespace lq2
