// Causal attention of a prefill step's new rows over the fp16 K/V of the same step, merged with the
// attention of the same rows over the pool-resident prefix (lq2_kv4_attention_prefix).
//
// The reference restores the prefix to fp16, concatenates it with the step's K/V and hands
// everything to flash-attn (qslab/runtime/model/attention.py:38-56,119-131).  Here the prefix is
// read as int4 by the KV4 kernels and this kernel adds the step's own part: row i of a sequence
// whose first row of the step is f attends to rows f..i, and the two parts are combined by their
// softmax weights,
//   out = (e^{m-M} acc + e^{lse_p-M} pre) / (e^{m-M} l + e^{lse_p-M}),  M = max(m, lse_p),
// (m, l, acc) being the running maximum, denominator and unnormalised sum of the own part and
// (pre, lse_p) the normalised output and log-sum-exp of the prefix part.
//
// A step's own part is small (64 batched tokens in chunked prefill), so the kernel is plain fp32 FMA
// work: one CTA per (row, KV head), one warp per query head of the group.  Scores: lane j of a warp
// takes key f + 32 t + j and walks its 2 D bytes against the query kept in shared memory as fp32.
// Values: the lanes split the channels and walk the 32 keys of the tile, the probability of each
// broadcast by shuffle.  Everything is in the base-2 domain.
#include "common.cuh"

namespace lq2 {
namespace {

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

template <int D>
__global__ void __launch_bounds__(256) chunk_attention_kernel(
    const __half* __restrict__ q, int64_t q_stride, const __half* __restrict__ k, int64_t k_stride,
    const __half* __restrict__ v, int64_t v_stride, const int32_t* __restrict__ first_row,
    const int32_t* __restrict__ prefix_row, const __half* __restrict__ pre, const float* __restrict__ pre_lse,
    __half* __restrict__ out, int hq, int hkv, float scale2) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int E = D / 32;                 // channels per lane in the value phase
    constexpr float kLog2e = 1.4426950408889634f;
    extern __shared__ __align__(16) float sq[];     // [rep][D]: the queries, scaled by D^-0.5 log2(e)
    const int row = blockIdx.x, kvh = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rep = hq / hkv, head = kvh * rep + warp;
    const int pr = prefix_row[row];
    if (pr < -1) return;                      // the caller computes this row elsewhere
    const int f = first_row[row];
    float* myq = sq + warp * D;
    const __half* qp = q + int64_t(row) * q_stride + head * D;
#pragma unroll
    for (int i = 0; i < E; ++i) myq[lane + 32 * i] = __half2float(qp[lane + 32 * i]) * scale2;
    __syncwarp();

    float m = -INFINITY, l = 0.f, acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    for (int base = f; base <= row; base += 32) {
        const int j = base + lane;
        float s = -INFINITY;
        if (j <= row) {
            const uint4* kp = reinterpret_cast<const uint4*>(k + int64_t(j) * k_stride + kvh * D);
            float d0 = 0.f, d1 = 0.f;
#pragma unroll 4
            for (int c = 0; c < D / 8; ++c) {
                const uint4 w = kp[c];
                const float4 qa = *reinterpret_cast<const float4*>(myq + 8 * c);
                const float4 qb = *reinterpret_cast<const float4*>(myq + 8 * c + 4);
                const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
                const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
                const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
                const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
                d0 += k0.x * qa.x + k0.y * qa.y + k1.x * qa.z + k1.y * qa.w;
                d1 += k2.x * qb.x + k2.y * qb.y + k3.x * qb.z + k3.y * qb.w;
            }
            s = d0 + d1;
        }
        float tm = s;
#pragma unroll
        for (int off = 16; off; off >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
        const float nm = fmaxf(m, tm);        // finite: key `base` is always within the row's range
        const float fac = ex2f(m - nm);
        const float p = j <= row ? ex2f(s - nm) : 0.f;
        float ps = p;
#pragma unroll
        for (int off = 16; off; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        l = l * fac + ps;
        m = nm;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] *= fac;
        const int n = min(32, row - base + 1);
        const __half* vp = v + int64_t(base) * v_stride + kvh * D + lane * E;
        for (int jj = 0; jj < n; ++jj) {
            const float pj = __shfl_sync(0xffffffffu, p, jj);
            const __half* vr = vp + int64_t(jj) * v_stride;
            if (E == 4) {
                const uint2 w = *reinterpret_cast<const uint2*>(vr);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
                acc[0] += pj * a.x; acc[1] += pj * a.y; acc[E - 2] += pj * b.x; acc[E - 1] += pj * b.y;
            } else {
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(vr));
                acc[0] += pj * a.x; acc[1] += pj * a.y;
            }
        }
    }

    // ---- merge with the prefix part
    float own = l, share = 0.f, fac = 1.f;
    const __half* pp = nullptr;
    if (pr >= 0) {
        const float lp = pre_lse[int64_t(pr) * hq + head] * kLog2e;
        if (lp > -INFINITY) {
            const float mm = fmaxf(m, lp);
            fac = ex2f(m - mm);
            own = l * fac;
            share = ex2f(lp - mm);
            pp = pre + (int64_t(pr) * hq + head) * D + lane * E;
        }
    }
    const float inv = 1.f / (own + share);
    __half* dst = out + (int64_t(row) * hq + head) * D + lane * E;
#pragma unroll
    for (int e = 0; e < E; e += 2) {
        float a = acc[e] * fac, b = acc[e + 1] * fac;
        if (pp) {
            const float2 t = __half22float2(*reinterpret_cast<const __half2*>(pp + e));
            a += share * t.x;
            b += share * t.y;
        }
        *reinterpret_cast<__half2*>(dst + e) = __floats2half2_rn(a * inv, b * inv);
    }
}

}  // namespace

int chunk_attention_launch(const __half* q, int64_t q_stride, const __half* k, int64_t k_stride, const __half* v,
                           int64_t v_stride, const int32_t* first_row, const int32_t* prefix_row,
                           const __half* pre, const float* pre_lse, __half* out, int rows, int hq, int hkv, int d,
                           cudaStream_t st) {
    const int rep = hq / hkv;
    const float scale2 = float(1.4426950408889634 / sqrt(double(d)));
    dim3 grid(rows, hkv), block(32 * rep);
    const size_t smem = size_t(rep) * d * sizeof(float);
    if (d == 128)
        return launch_pdl(chunk_attention_kernel<128>, grid, block, smem, st, 1, q, q_stride, k, k_stride, v, v_stride,
                          first_row, prefix_row, pre, pre_lse, out, hq, hkv, scale2);
    return launch_pdl(chunk_attention_kernel<64>, grid, block, smem, st, 1, q, q_stride, k, k_stride, v, v_stride,
                      first_row, prefix_row, pre, pre_lse, out, hq, hkv, scale2);
}

}  // namespace lq2
