// Sum all-reduce of a small fp16 activation tensor across the tensor-parallel ranks of one
// NVSwitch domain, as one kernel per rank over peer memory (no library collective).
//
// The reference is single-GPU (qslab/runtime/model/qwen3.py:1-5); this is the exchange the
// row-split o_proj / down_proj gain under tensor parallelism: two [M, hidden] fp16 sums per
// decoder layer, 256 KB each at batch 32, where a library all-reduce is all latency.
//
// Every rank owns one exchange buffer allocated with cudaMalloc and mapped into the other
// ranks through CUDA IPC:
//     calls, done                          u32   calls completed by this rank; CTAs finished in the
//                                                running call (the last one advances `calls`)
//     flags    [2][world][kMaxCtas]        u32   flags[q][src][b] = sequence number of the last
//                                                call of parity q whose slice b arrived from src
//     slots    [2][world][max_bytes]       fp16  slots[q][src] = src's addend for that call
//     llslots  [2][world][2 * max_bytes]         the same addends in flagged form (see below)
// Every rank issues the same calls in the same order on one stream, so the call's sequence
// number (calls + 1, read after the previous kernel has completed) and its parity q agree on
// all ranks without any host state, also when the launches are replayed from a CUDA graph.
// One call: CTA b of rank r owns a fixed slice of the tensor.  It (1) stores its slice of x
// into slots[q][r] of every peer with plain peer stores, (2) after a system-scope fence
// writes the call's sequence number into flags[q][r][b] of every peer, (3) waits until its
// own flags[q][src][b] show that number for every src, (4) adds the addends in rank order
// in fp32 (its own straight from x), so every rank obtains the same bits, and writes fp16.
// A CTA only ever waits for the same CTA of its peers, so no grid-wide barrier exists, and
// the two parities make a slot reusable: consecutive calls use different halves, and a peer
// can only start call c+2 after it has seen this rank's flags of call c+1, which this rank
// sends after call c has completed.
//
// Fused form (lq2_rmsnorm_allreduce): the all-reduce that precedes a residual RMSNorm is done
// inside the norm kernel, so the exchange costs no launch of its own.  A CTA owns whole rows.
// Each thread stores its 16-byte chunk of the local addend into llslots[q][r] of every peer
// as two 16-byte words {data, seq, data, seq}: every 8 bytes carry their own copy of the
// call's sequence number, so the receiver needs no separate flag and the sender no fence - it
// polls the chunk itself until all four numbers match, one NVLink crossing in total.
//
// Every wait is bounded.  A thread has one budget of polls for the whole kernel (the limit set
// with lq2_allreduce_set_poll_limit, a kernel argument), shared by all the chunks and peers it
// waits for: once it is spent the thread stops waiting, the failure is counted in
// g_lq2_allreduce_timeouts and the kernel finishes with whatever it has, so a missing peer
// costs one budget, not one per wait, and cannot hang the GPU.  The host reads the counter
// with lq2_allreduce_timeouts().
#include <cstring>

#include "common.cuh"

namespace lq2 {

namespace {

constexpr int kArThreads = 512;
constexpr int kBytesPerCta = kArThreads * 16;          // one 128-bit access per thread and pass
constexpr long long kDefaultPollLimit = 1ll << 22;      // a few seconds of polling per thread

__device__ unsigned int g_lq2_allreduce_timeouts = 0;

__device__ __forceinline__ unsigned int ld_volatile_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.volatile.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_volatile_u4(const void* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void add8(float (&acc)[8], const uint4& v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(u32_as_h2(w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
    }
}

__global__ void __launch_bounds__(kArThreads) tp_allreduce_kernel(const __half* x, __half* out,
                                                                  const PeerTable peers, const int rank,
                                                                  const int world, const size_t bytes,
                                                                  const size_t max_bytes, const long long poll_limit) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ unsigned int s_seq;
    const int b = blockIdx.x, tid = threadIdx.x;
    unsigned char* mine = peer_base(peers, rank);
    unsigned int* calls = reinterpret_cast<unsigned int*>(mine);
    unsigned int* done = calls + 1;
    if (tid == 0) s_seq = *calls + 1;
    __syncthreads();
    const unsigned int seq = s_seq;
    const int q = int(seq & 1u);
    const size_t slots = slots_offset(world);
    // slice of this CTA: 16-byte units [u0, u1)
    const size_t units = bytes / 16;
    const size_t per = (units + gridDim.x - 1) / gridDim.x;
    const size_t u0 = min(units, size_t(b) * per), u1 = min(units, u0 + per);
    const uint4* x4 = reinterpret_cast<const uint4*>(x);

    // (1) my addend into every peer's slot
    for (size_t u = u0 + tid; u < u1; u += kArThreads) {
        const uint4 v = x4[u];
        for (int p = 0; p < world; ++p) {
            if (p == rank) continue;
            uint4* dst = reinterpret_cast<uint4*>(peer_base(peers, p) + slots + (size_t(q) * world + rank) * max_bytes);
            dst[u] = v;
        }
    }
    __threadfence_system();
    __syncthreads();
    // (2) tell every peer, (3) wait for every peer
    if (tid < world && tid != rank) {
        unsigned int* theirs = reinterpret_cast<unsigned int*>(peer_base(peers, tid) + flags_offset()) +
                               (size_t(q) * world + rank) * kMaxCtas + b;
        st_release_sys(theirs, seq);
        const unsigned int* own = reinterpret_cast<const unsigned int*>(mine + flags_offset()) +
                                  (size_t(q) * world + tid) * kMaxCtas + b;
        long long polls = 0;
        while (ld_acquire_sys(own) != seq) {
            if (++polls >= poll_limit) {
                atomicAdd(&g_lq2_allreduce_timeouts, 1u);
                break;
            }
        }
    }
    __syncthreads();
    // (4) sum in rank order
    uint4* out4 = reinterpret_cast<uint4*>(out);
    for (size_t u = u0 + tid; u < u1; u += kArThreads) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < world; ++p) {
            if (p == rank) {
                add8(acc, x4[u]);
            } else {
                const uint4* src = reinterpret_cast<const uint4*>(mine + slots + (size_t(q) * world + p) * max_bytes);
                add8(acc, ld_volatile_u4(src + u));
            }
        }
        uint4 r;
        r.x = h2_as_u32(__floats2half2_rn(acc[0], acc[1]));
        r.y = h2_as_u32(__floats2half2_rn(acc[2], acc[3]));
        r.z = h2_as_u32(__floats2half2_rn(acc[4], acc[5]));
        r.w = h2_as_u32(__floats2half2_rn(acc[6], acc[7]));
        out4[u] = r;
    }
    // the last CTA of the call advances the rank's call counter for the next launch
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            *calls = seq;
        }
    }
}

// ---------------------------------------------------------------- all-reduce + residual RMSNorm
constexpr int kNormThreads = 256;     // thread count and chunk order of rmsnorm_kernel: the two must round alike
constexpr int kNormMaxChunks = 4;     // 8 halves per chunk per thread: hidden <= 8192

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// h = fp16(sum over ranks of x_r) (rank order, fp32), then exactly the residual RMSNorm of
// qslab/runtime/model/primitives.py:23-30 on h: s = fp32(h) + fp32(residual),
// residual_out = fp16(s), out = fp16(s * rsqrt(mean(s^2) + eps)) * weight.
// CH: chunks per thread this instantiation provides for (hidden <= 2048 * CH); W: ranks it provides for.
// Both bound the registers that hold peers' words in flight: the kernel shares its SM with the CTAs of the
// next projection, which programmatic dependent launch brings in early, so a fat CTA here delays them
// (218 registers per thread cost 7 % of a two-GPU decode step).
template <int CH, int W>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_allreduce_kernel(
    const __half* x, int64_t x_stride, const __half* residual, const __half* __restrict__ weight, __half* out,
    __half* residual_out, const int hidden, const float eps, const PeerTable peers, const int rank,
    const int world, const size_t max_bytes, const int pushed, const long long poll_limit) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float partial[kNormThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    unsigned char* mine = peer_base(peers, rank);
    unsigned int* calls = reinterpret_cast<unsigned int*>(mine);
    unsigned int* done = calls + 1;
    const int chunks = hidden / 8;
    // Everything that does not depend on the call's sequence number is requested at once - the number itself
    // (every thread reads it: the last CTA of a call advances it only after all CTAs have arrived at the end),
    // this rank's addend, the residual and the norm weight - so that the kernel is two memory round trips
    // (these, then the peers' words) instead of one per operand.
    const unsigned int seq = ld_volatile_u32(calls) + 1;
    uint4 own[CH], res_w[CH], norm_w[CH];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int idx = tid + c * kNormThreads;
        if (idx < chunks) {
            own[c] = *reinterpret_cast<const uint4*>(x + int64_t(row) * x_stride + idx * 8);
            res_w[c] = *reinterpret_cast<const uint4*>(residual + int64_t(row) * hidden + idx * 8);
            norm_w[c] = *reinterpret_cast<const uint4*>(weight + idx * 8);
        }
    }
    const size_t ll = llslots_offset(world, max_bytes) + size_t(seq & 1u) * world * 2 * max_bytes;

    // the flagged copy of my addend into every peer
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int idx = tid + c * kNormThreads;
        if (idx < chunks) {
            const uint4 lo = make_uint4(own[c].x, seq, own[c].y, seq), hi = make_uint4(own[c].z, seq, own[c].w, seq);
            const size_t off = ll + size_t(rank) * 2 * max_bytes + (size_t(row) * chunks + idx) * 32;
            for (int p = 0; p < world; ++p) {
                if (p == rank || pushed) continue;          // pushed: the producing kernel has sent it already
                uint4* dst = reinterpret_cast<uint4*>(peer_base(peers, p) + off);
                dst[0] = lo;
                dst[1] = hi;
            }
        }
    }
    // gather, sum in rank order, residual add.  All peers' words of all of this thread's chunks are requested
    // before the first one is examined: looked at one after the other, the round trips of a thread add up
    // (14 in a row at eight ranks with two chunks per thread), which is what an exchange used to cost there.
    float v[CH][8];
    float ss = 0.f;
    bool gave_up = false;
    long long budget = poll_limit;                      // polls left to this thread, over all its waits
    // Words in flight per thread: at most eight peer entries (64 registers), taken as whole chunks when the
    // ranks are few and as groups of four peers of one chunk when they are many.
    constexpr int G = W < 4 ? W : 4;                     // peers requested together
    constexpr int AHEAD = CH * W <= 8 ? CH : (2 * W <= 8 && CH >= 2 ? 2 : 1);   // chunks requested together
    uint4 lo[AHEAD][G], hi[AHEAD][G];
    auto request = [&](int c, int slot, int p0) {
        const int idx = tid + c * kNormThreads;
        if (idx >= chunks) return;
        const unsigned char* base = mine + ll + (size_t(row) * chunks + idx) * 32;
#pragma unroll
        for (int j = 0; j < G; ++j) {
            const int p = p0 + j;
            if (p < world && p != rank) {
                lo[slot][j] = ld_volatile_u4(base + size_t(p) * 2 * max_bytes);
                hi[slot][j] = ld_volatile_u4(base + size_t(p) * 2 * max_bytes + 16);
            }
        }
    };
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int idx = tid + c * kNormThreads;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int p0 = 0; p0 < W; p0 += G) {
            if (W <= G) {                                // all peers fit: the next AHEAD chunks at once
                if (c % AHEAD == 0) {
#pragma unroll
                    for (int a = 0; a < AHEAD; ++a)
                        if (c + a < CH) request(c + a, a, 0);
                }
            } else {
                request(c, 0, p0);
            }
            if (idx < chunks) {
                const int slot = W <= G ? c % AHEAD : 0;
                const unsigned char* base = mine + ll + (size_t(row) * chunks + idx) * 32;
#pragma unroll
                for (int j = 0; j < G; ++j) {
                    const int p = p0 + j;
                    if (p >= world) continue;
                    if (p == rank) {
                        add8(acc, own[c]);
                        continue;
                    }
                    const unsigned char* src = base + size_t(p) * 2 * max_bytes;
                    uint4 a = lo[slot][j], b = hi[slot][j];
                    while (!(a.y == seq && a.w == seq && b.y == seq && b.w == seq)) {
                        if (--budget <= 0) {            // spent: this and every later wait ends after one look
                            gave_up = true;
                            break;
                        }
                        a = ld_volatile_u4(src);
                        b = ld_volatile_u4(src + 16);
                    }
                    add8(acc, make_uint4(a.x, a.z, b.x, b.z));
                }
            }
        }
        if (idx < chunks) {
            const __half2* r = reinterpret_cast<const __half2*>(&res_w[c]);
            __half2 o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 h = __half22float2(__floats2half2_rn(acc[2 * i], acc[2 * i + 1]));   // the all-reduced fp16
                const float2 b = __half22float2(r[i]);
                v[c][2 * i] = h.x + b.x;
                v[c][2 * i + 1] = h.y + b.y;
                ss += v[c][2 * i] * v[c][2 * i] + v[c][2 * i + 1] * v[c][2 * i + 1];
                o[i] = __floats2half2_rn(v[c][2 * i], v[c][2 * i + 1]);
            }
            *reinterpret_cast<uint4*>(residual_out + int64_t(row) * hidden + idx * 8) = *reinterpret_cast<uint4*>(o);
        }
    }
    if (gave_up) atomicAdd(&g_lq2_allreduce_timeouts, 1u);
    ss = warp_sum(ss);
    if ((tid & 31) == 0) partial[tid >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) total += partial[w];
    const float rs = rsqrtf(total / float(hidden) + eps);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
        const int idx = tid + c * kNormThreads;
        if (idx < chunks) {
            const __half2* w = reinterpret_cast<const __half2*>(&norm_w[c]);
            __half2 o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                o[i] = __hmul2(__floats2half2_rn(v[c][2 * i] * rs, v[c][2 * i + 1] * rs), w[i]);
            *reinterpret_cast<uint4*>(out + int64_t(row) * hidden + idx * 8) = *reinterpret_cast<uint4*>(o);
        }
    }
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0;
            *calls = seq;
        }
    }
}

}  // namespace

}  // namespace lq2

using namespace lq2;

#include <atomic>

namespace {
std::atomic<long long> g_poll_limit{kDefaultPollLimit};
}  // namespace

extern "C" {

long long lq2_allreduce_set_poll_limit(long long polls) {
    return g_poll_limit.exchange(polls > 0 ? polls : kDefaultPollLimit, std::memory_order_relaxed);
}

size_t lq2_allreduce_buffer_bytes(int world, size_t max_message_bytes) {
    if (world < 2 || world > kMaxWorld || max_message_bytes == 0 || max_message_bytes % 16) return 0;
    return llslots_offset(world, max_message_bytes) + size_t(4) * world * max_message_bytes;
}

int lq2_allreduce_buffer_create(size_t bytes, void** buffer, void* ipc_handle_64) {
    if (!buffer || !ipc_handle_64 || bytes == 0) return LQ2_ERR_ARG;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return LQ2_ERR_CUDA;
    if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p);
        return LQ2_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return LQ2_ERR_CUDA;
    }
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    memcpy(ipc_handle_64, &h, 64);
    *buffer = p;
    return LQ2_OK;
}

int lq2_allreduce_buffer_open(const void* ipc_handle_64, void** buffer) {
    if (!ipc_handle_64 || !buffer) return LQ2_ERR_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle_64, 64);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return LQ2_ERR_CUDA;
    }
    *buffer = p;
    return LQ2_OK;
}

int lq2_allreduce_buffer_close(void* buffer, int own) {
    if (!buffer) return LQ2_OK;
    const cudaError_t e = own ? cudaFree(buffer) : cudaIpcCloseMemHandle(buffer);
    return e == cudaSuccess ? LQ2_OK : LQ2_ERR_CUDA;
}

unsigned int lq2_allreduce_timeouts(void) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_lq2_allreduce_timeouts, sizeof(v)) != cudaSuccess) return ~0u;
    return v;
}

int lq2_allreduce_fp16(const void* x, void* out, int64_t count, void* const* buffers, int rank, int world,
                       size_t max_message_bytes, void* stream) {
    if (count == 0) return LQ2_OK;
    if (!x || !out || !buffers || count < 0) return LQ2_ERR_ARG;
    if (world < 2 || world > kMaxWorld || rank < 0 || rank >= world) return LQ2_ERR_SHAPE;
    const size_t bytes = size_t(count) * 2;
    if (bytes % 16 || max_message_bytes % 16) return LQ2_ERR_SHAPE;
    if (bytes > max_message_bytes) return LQ2_ERR_LIMIT;
    if (!aligned(x, 16) || !aligned(out, 16)) return LQ2_ERR_ALIGN;
    PeerTable peers;
    for (int p = 0; p < kMaxWorld; ++p) {
        peers.base[p] = p < world ? static_cast<unsigned char*>(buffers[p]) : nullptr;
        if (p < world && !peers.base[p]) return LQ2_ERR_ARG;
    }
    // The grid is a function of the message size only, so every rank launches the same
    // CTAs for the same call (the per-CTA sequence numbers depend on it).
    int grid = int((bytes + kBytesPerCta - 1) / kBytesPerCta);
    if (grid > kMaxCtas) grid = kMaxCtas;
    return launch_pdl(tp_allreduce_kernel, dim3(grid), dim3(kArThreads), 0, static_cast<cudaStream_t>(stream), 1,
                      static_cast<const __half*>(x), static_cast<__half*>(out), peers, rank, world, bytes,
                      max_message_bytes, g_poll_limit.load(std::memory_order_relaxed));
}

static int rmsnorm_allreduce_impl(const void* x, int64_t x_row_stride, const void* residual, const void* weight,
                                  void* out, void* residual_out, int rows, int hidden, float eps, void* const* buffers,
                                  int rank, int world, size_t max_message_bytes, int pushed, void* stream) {
    if (rows == 0) return LQ2_OK;
    if (!x || !residual || !weight || !out || !residual_out || !buffers || rows < 0 || hidden <= 0) return LQ2_ERR_ARG;
    if (world < 2 || world > kMaxWorld || rank < 0 || rank >= world) return LQ2_ERR_SHAPE;
    if (hidden % 8 || hidden > 8 * kNormThreads * kNormMaxChunks || max_message_bytes % 16) return LQ2_ERR_SHAPE;
    if (size_t(rows) * hidden * 2 > max_message_bytes) return LQ2_ERR_LIMIT;
    if (!aligned(x, 16) || x_row_stride % 8 || !aligned(weight, 16) || !aligned(out, 16) || !aligned(residual, 16) ||
        !aligned(residual_out, 16))
        return LQ2_ERR_ALIGN;
    PeerTable peers;
    for (int p = 0; p < kMaxWorld; ++p) {
        peers.base[p] = p < world ? static_cast<unsigned char*>(buffers[p]) : nullptr;
        if (p < world && !peers.base[p]) return LQ2_ERR_ARG;
    }
    auto launch = [&](auto kernel) {
        return launch_pdl(kernel, dim3(rows), dim3(kNormThreads), 0, static_cast<cudaStream_t>(stream), 1,
                          static_cast<const __half*>(x), x_row_stride, static_cast<const __half*>(residual),
                          static_cast<const __half*>(weight), static_cast<__half*>(out),
                          static_cast<__half*>(residual_out), hidden, eps, peers, rank, world, max_message_bytes,
                          pushed, g_poll_limit.load(std::memory_order_relaxed));
    };
    const int ch = hidden <= 8 * kNormThreads ? 1 : (hidden <= 16 * kNormThreads ? 2 : 4);
    if (world <= 2) return ch == 1 ? launch(rmsnorm_allreduce_kernel<1, 2>) : ch == 2 ? launch(rmsnorm_allreduce_kernel<2, 2>) : launch(rmsnorm_allreduce_kernel<4, 2>);
    if (world <= 4) return ch == 1 ? launch(rmsnorm_allreduce_kernel<1, 4>) : ch == 2 ? launch(rmsnorm_allreduce_kernel<2, 4>) : launch(rmsnorm_allreduce_kernel<4, 4>);
    return ch == 1 ? launch(rmsnorm_allreduce_kernel<1, 8>) : ch == 2 ? launch(rmsnorm_allreduce_kernel<2, 8>) : launch(rmsnorm_allreduce_kernel<4, 8>);
}

int lq2_rmsnorm_allreduce(const void* x, int64_t x_row_stride, const void* residual, const void* weight, void* out,
                          void* residual_out, int rows, int hidden, float eps, void* const* buffers, int rank,
                          int world, size_t max_message_bytes, void* stream) {
    return rmsnorm_allreduce_impl(x, x_row_stride, residual, weight, out, residual_out, rows, hidden, eps, buffers, rank,
                                  world, max_message_bytes, 0, stream);
}

int lq2_rmsnorm_allreduce_pushed(const void* x, int64_t x_row_stride, const void* residual, const void* weight,
                                 void* out, void* residual_out, int rows, int hidden, float eps, void* const* buffers,
                                 int rank, int world, size_t max_message_bytes, void* stream) {
    return rmsnorm_allreduce_impl(x, x_row_stride, residual, weight, out, residual_out, rows, hidden, eps, buffers, rank,
                                  world, max_message_bytes, 1, stream);
}

}  // extern "C"
