// Fused elementwise operators around the W4A16 and KV4 kernels.
//
// The reference runs these steps as separate eager torch kernels, about fifty
// launches per decoder layer:
//   RMSNorm with optional residual add     qslab/runtime/model/primitives.py:15-30
//   q/k RMSNorm, RoPE                      qslab/runtime/model/qwen3.py:49-51, rotary.py:12-16,103-108
//   SmoothAttention scaling                qslab/runtime/model/attention.py:72-77
//   KV4 store                              qslab/kernels/kv4/store.py:9-68
//   SiLU(gate) * up                        qslab/runtime/model/qwen3.py:64
// Each kernel below keeps the reference's rounding points: statistics and
// rotations in fp32, a cast to fp16 after the normalisation, fp16 products with
// the norm weight and with lambda, fp16 result of SiLU before the product.
#include <algorithm>

#include "common.cuh"

namespace lq2 {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- RMSNorm
// One CTA per row.  With a residual: s = x + residual in fp32, residual_out =
// fp16(s), statistics over the unrounded s (primitives.py:23-28).
constexpr int kNormThreads = 256;
constexpr int kNormMaxChunks = 4;     // 8 halves per chunk per thread: hidden <= 8192

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(
    const __half* __restrict__ x, int64_t x_stride, const __half* __restrict__ residual,
    const __half* __restrict__ weight, __half* __restrict__ out, __half* __restrict__ residual_out,
    int hidden, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float partial[kNormThreads / 32];
    const int row = blockIdx.x, tid = threadIdx.x;
    const int chunks = hidden / 8;
    float v[kNormMaxChunks][8];
    float ss = 0.f;
    // the norm weights are requested with the inputs, not after the reduction: one memory round trip less
    uint4 norm_w[kNormMaxChunks];
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
        const int idx = tid + c * kNormThreads;
        if (idx < chunks) norm_w[c] = *reinterpret_cast<const uint4*>(weight + idx * 8);
    }
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
        const int idx = tid + c * kNormThreads;
        if (idx < chunks) {
            const uint4 raw = *reinterpret_cast<const uint4*>(x + int64_t(row) * x_stride + idx * 8);
            const __half2* h = reinterpret_cast<const __half2*>(&raw);
            uint4 rr = make_uint4(0, 0, 0, 0);
            if (residual) rr = *reinterpret_cast<const uint4*>(residual + int64_t(row) * hidden + idx * 8);
            const __half2* r = reinterpret_cast<const __half2*>(&rr);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 a = __half22float2(h[i]);
                if (residual) {
                    const float2 b = __half22float2(r[i]);
                    a.x += b.x;
                    a.y += b.y;
                }
                v[c][2 * i] = a.x;
                v[c][2 * i + 1] = a.y;
                ss += a.x * a.x + a.y * a.y;
            }
            if (residual_out) {
                __half2 o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) o[i] = __floats2half2_rn(v[c][2 * i], v[c][2 * i + 1]);
                *reinterpret_cast<uint4*>(residual_out + int64_t(row) * hidden + idx * 8) = *reinterpret_cast<uint4*>(o);
            }
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) partial[tid >> 5] = ss;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) total += partial[w];
    const float r = rsqrtf(total / float(hidden) + eps);
#pragma unroll
    for (int c = 0; c < kNormMaxChunks; ++c) {
        const int idx = tid + c * kNormThreads;
        if (idx < chunks) {
            const __half2* w = reinterpret_cast<const __half2*>(&norm_w[c]);
            __half2 o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                o[i] = __hmul2(__floats2half2_rn(v[c][2 * i] * r, v[c][2 * i + 1] * r), w[i]);
            *reinterpret_cast<uint4*>(out + int64_t(row) * hidden + idx * 8) = *reinterpret_cast<uint4*>(o);
        }
    }
}

// ---------------------------------------------------------------- SiLU * up
__global__ void __launch_bounds__(256) silu_mul_kernel(const __half* __restrict__ gate, int64_t g_stride,
                                                       const __half* __restrict__ up, int64_t u_stride,
                                                       __half* __restrict__ out, int rows, int width) {
    pdl_launch_dependents();
    pdl_wait();
    const int chunks = width / 8;
    const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= int64_t(rows) * chunks) return;
    const int row = int(id / chunks), c = int(id % chunks);
    const uint4 gr = *reinterpret_cast<const uint4*>(gate + int64_t(row) * g_stride + c * 8);
    const uint4 ur = *reinterpret_cast<const uint4*>(up + int64_t(row) * u_stride + c * 8);
    const __half2* g = reinterpret_cast<const __half2*>(&gr);
    const __half2* u = reinterpret_cast<const __half2*>(&ur);
    __half2 o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = silu_mul2(g[i], u[i]);
    *reinterpret_cast<uint4*>(out + (int64_t(row) * chunks + c) * 8) = *reinterpret_cast<uint4*>(o);
}

// ------------------------------------------- q/k norm + RoPE + lambda + KV4 store
// One warp per (token, head); heads 0..HQ-1 are query heads, HQ..HQ+HKV-1 key
// heads (which also carry the value head of the same index).  Lane l holds
// channels EPL*l .. EPL*l+EPL-1 of the first half and the same offsets of the
// second half, so a rotation pair (d, d + D/2) lives in one lane.
struct PreAttnParams {
    const __half* q; const __half* k; const __half* v;
    int64_t q_stride, k_stride, v_stride;
    const __half* q_weight; const __half* k_weight;
    const float* cos_sin;            // [max_pos, D]: cos (D/2) then sin (D/2)
    const int64_t* positions;
    const __half* lam_q; const __half* lam_k;   // optional [HQ, D], [HKV, D]
    __half* q_out; __half* k_out;    // [T, HQ, D] ; optional [T, HKV, D]
    uint32_t* kq; const __half* ks; uint32_t* vq; __half* vs;
    const int32_t* slots;            // null: no store
    int tokens, hq, hkv, v_group;
    int64_t num_slots;
    float eps;
};

__device__ __forceinline__ uint32_t kv_code(float x, float s) {
    const float q = floorf(fminf(fmaxf(__fdiv_rn(x, s), -8.0f), 7.0f) + 0.5f);
    return uint32_t(int(q) + 8) & 15u;
}

template <int D>
__global__ void __launch_bounds__(128) pre_attention_kernel(const PreAttnParams p) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int EPL = D / 64;              // elements per lane per half
    constexpr int HALF = D / 2;
    constexpr int LPW = 8 / EPL;             // lanes per packed word
    const int lane = threadIdx.x & 31;
    const int64_t wid = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int heads = p.hq + p.hkv;
    if (wid >= int64_t(p.tokens) * heads) return;
    const int token = int(wid / heads), head = int(wid % heads);
    const bool is_q = head < p.hq;
    const int h = is_q ? head : head - p.hq;
    const __half* src = is_q ? p.q + int64_t(token) * p.q_stride + h * D : p.k + int64_t(token) * p.k_stride + h * D;
    const __half* wgt = is_q ? p.q_weight : p.k_weight;
    const int d0 = EPL * lane;

    // Everything whose address is known now is requested now - the position (the rotation table row
    // depends on it), the pool slot and the value row of a key head, the norm weights - so that the
    // kernel is two memory round trips, not one per operand.
    const int64_t position = p.positions[token];
    const bool kv_head = !is_q && p.slots != nullptr;
    const int64_t slot = kv_head ? int64_t(p.slots[token]) : -1;
    float a[EPL], b[EPL];                    // first half, second half
    float va[EPL], vb[EPL];
    __half wa[EPL], wb[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        a[i] = __half2float(src[d0 + i]);
        b[i] = __half2float(src[HALF + d0 + i]);
        wa[i] = wgt[d0 + i];
        wb[i] = wgt[HALF + d0 + i];
    }
    if (kv_head) {
        const __half* vsrc = p.v + int64_t(token) * p.v_stride + h * D;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            va[i] = __half2float(vsrc[d0 + i]);
            vb[i] = __half2float(vsrc[HALF + d0 + i]);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) ss += a[i] * a[i] + b[i] * b[i];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / float(D) + p.eps);
    const float* cs = p.cos_sin + position * D;
    __half oa[EPL], ob[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        // norm -> fp16, * weight in fp16, rotation in fp32 -> fp16
        const float x1 = __half2float(__hmul(__float2half_rn(a[i] * r), wa[i]));
        const float x2 = __half2float(__hmul(__float2half_rn(b[i] * r), wb[i]));
        const float c = cs[d0 + i], s = cs[HALF + d0 + i];
        oa[i] = __float2half_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s)));
        ob[i] = __float2half_rn(__fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s)));
    }
    if (is_q) {
        __half* dst = p.q_out + (int64_t(token) * p.hq + h) * D;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            if (p.lam_q) {
                oa[i] = __hmul(oa[i], p.lam_q[h * D + d0 + i]);
                ob[i] = __hmul(ob[i], p.lam_q[h * D + HALF + d0 + i]);
            }
            dst[d0 + i] = oa[i];
            dst[HALF + d0 + i] = ob[i];
        }
        return;
    }
    // ---- key head: lambda division, optional fp16 copy, then quantize K and V of this head
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        if (p.lam_k) {   // fp16 / fp16 evaluated in fp32 and rounded once, as torch does
            oa[i] = __float2half_rn(__fdiv_rn(__half2float(oa[i]), __half2float(p.lam_k[h * D + d0 + i])));
            ob[i] = __float2half_rn(__fdiv_rn(__half2float(ob[i]), __half2float(p.lam_k[h * D + HALF + d0 + i])));
        }
        if (p.k_out) {
            __half* dst = p.k_out + (int64_t(token) * p.hkv + h) * D;
            dst[d0 + i] = oa[i];
            dst[HALF + d0 + i] = ob[i];
        }
    }
    if (!p.slots) return;
    const bool write = slot >= 0 && slot < p.num_slots;
    float m1 = 0.f, m2 = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        m1 = fmaxf(m1, fabsf(va[i]));
        m2 = fmaxf(m2, fabsf(vb[i]));
    }
    // amax over each value group: lanes_per_group lanes of one half, or the whole row
    const int lanes_per_group = p.v_group / EPL;          // 16, 32 or 64 (= both halves)
    if (lanes_per_group > 32) { m1 = fmaxf(m1, m2); m2 = m1; }
    for (int o = 1; o < min(lanes_per_group, 32); o <<= 1) {
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
        m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
    }
    if (lanes_per_group > 32) { m1 = fmaxf(m1, m2); m2 = m1; }
    const float s1 = fmaxf(__fdiv_rn(m1, 7.0f), 1e-4f), s2 = fmaxf(__fdiv_rn(m2, 7.0f), 1e-4f);
    const __half* ksp = p.ks + h * D;
    uint32_t kw1 = 0, kw2 = 0, vw1 = 0, vw2 = 0;
    const int nib0 = (lane % LPW) * EPL;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int sh = 4 * (nib0 + i);
        kw1 |= kv_code(__half2float(oa[i]), __half2float(ksp[d0 + i])) << sh;
        kw2 |= kv_code(__half2float(ob[i]), __half2float(ksp[HALF + d0 + i])) << sh;
        vw1 |= kv_code(va[i], s1) << sh;
        vw2 |= kv_code(vb[i], s2) << sh;
    }
    for (int o = 1; o < LPW; o <<= 1) {
        kw1 |= __shfl_xor_sync(0xffffffffu, kw1, o);
        kw2 |= __shfl_xor_sync(0xffffffffu, kw2, o);
        vw1 |= __shfl_xor_sync(0xffffffffu, vw1, o);
        vw2 |= __shfl_xor_sync(0xffffffffu, vw2, o);
    }
    if (!write) return;
    constexpr int NW = D / 8;
    const int64_t base = (slot * p.hkv + h) * NW;
    if (lane % LPW == 0) {
        const int w = lane / LPW;
        p.kq[base + w] = kw1;
        p.kq[base + NW / 2 + w] = kw2;
        p.vq[base + w] = vw1;
        p.vq[base + NW / 2 + w] = vw2;
    }
    const int ng = D / p.v_group;
    __half* vsd = p.vs + (slot * p.hkv + h) * ng;
    if (ng == 1) {
        if (lane == 0) vsd[0] = __float2half_rn(s1);
    } else {
        // groups of the first half start at lanes 0, lpg, ...; second half likewise
        if (lane % lanes_per_group == 0) {
            vsd[lane / lanes_per_group] = __float2half_rn(s1);
            vsd[ng / 2 + lane / lanes_per_group] = __float2half_rn(s2);
        }
    }
}

// ---------------------------------------------------------------- decode step staging
// One launch fills the fixed input buffers of a captured decode graph from one packed
// int32 record [ids | positions | slots | context lens | block tables (batch x width)],
// including the padding of the unused rows (slot -1, context length 0, table 0), which
// the reference does with seven small device copies (cuda_graph.py:60-72).
__global__ void __launch_bounds__(256) stage_decode_kernel(const int32_t* __restrict__ packed, int64_t* input_ids,
                                                           int64_t* positions, int32_t* slot_mapping,
                                                           int32_t* context_lens, int32_t* block_tables,
                                                           int batch, int rows_cap, int width, int width_cap) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int total = rows_cap * width_cap;
    if (i < rows_cap) {
        const bool live = i < batch;
        if (live) {
            input_ids[i] = packed[i];
            positions[i] = packed[batch + i];
        }
        slot_mapping[i] = live ? packed[2 * batch + i] : -1;
        context_lens[i] = live ? packed[3 * batch + i] : 0;
    }
    if (i < total) {
        const int r = i / width_cap, c = i - r * width_cap;
        block_tables[i] = (r < batch && c < width) ? packed[4 * batch + r * width + c] : 0;
    }
}

}  // namespace
}  // namespace lq2

using namespace lq2;

extern "C" {

int lq2_rmsnorm(const void* x, int64_t x_row_stride, const void* residual, const void* weight, void* out,
                void* residual_out, int rows, int hidden, float eps, void* stream) {
    if (rows == 0) return LQ2_OK;
    if (!x || !weight || !out || rows < 0 || hidden <= 0) return LQ2_ERR_ARG;
    if (hidden % 8 || hidden > 8 * kNormThreads * kNormMaxChunks || (residual_out && !residual)) return LQ2_ERR_SHAPE;
    if (!aligned(x, 16) || x_row_stride % 8 || !aligned(weight, 16) || !aligned(out, 16) ||
        (residual && !aligned(residual, 16)) || (residual_out && !aligned(residual_out, 16)))
        return LQ2_ERR_ALIGN;
    return launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, static_cast<cudaStream_t>(stream), 1,
                      static_cast<const __half*>(x), x_row_stride, static_cast<const __half*>(residual),
                      static_cast<const __half*>(weight), static_cast<__half*>(out),
                      static_cast<__half*>(residual_out), hidden, eps);
}

int lq2_silu_mul(const void* gate, int64_t gate_row_stride, const void* up, int64_t up_row_stride, void* out,
                 int rows, int width, void* stream) {
    if (rows == 0) return LQ2_OK;
    if (!gate || !up || !out || rows < 0 || width <= 0) return LQ2_ERR_ARG;
    if (width % 8) return LQ2_ERR_SHAPE;
    if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(out, 16) || gate_row_stride % 8 || up_row_stride % 8)
        return LQ2_ERR_ALIGN;
    const int64_t total = int64_t(rows) * (width / 8);
    return launch_pdl(silu_mul_kernel, dim3(unsigned(cdiv64(total, 256))), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), 1, static_cast<const __half*>(gate), gate_row_stride,
                      static_cast<const __half*>(up), up_row_stride, static_cast<__half*>(out), rows, width);
}

int lq2_pre_attention(const void* q, const void* k, const void* v, int64_t q_stride, int64_t k_stride,
                      int64_t v_stride, const void* q_norm_weight, const void* k_norm_weight,
                      const float* cos_sin, const int64_t* positions, const void* lam_q, const void* lam_k,
                      void* q_out, void* k_out, uint32_t* kq, const void* ks, uint32_t* vq, void* vs,
                      const int32_t* slots, int tokens, int hq, int hkv, int d, int v_group, int64_t num_slots,
                      float eps, void* stream) {
    if (tokens == 0) return LQ2_OK;
    if (!q || !k || !q_norm_weight || !k_norm_weight || !cos_sin || !positions || !q_out || tokens < 0 ||
        hq <= 0 || hkv <= 0)
        return LQ2_ERR_ARG;
    if (d != 64 && d != 128) return LQ2_ERR_SHAPE;
    if (slots) {
        if (!v || !kq || !ks || !vq || !vs || num_slots <= 0) return LQ2_ERR_ARG;
        if (v_group < 8 || (v_group & (v_group - 1)) || d % v_group) return LQ2_ERR_SHAPE;
    }
    PreAttnParams p;
    p.q = static_cast<const __half*>(q); p.k = static_cast<const __half*>(k); p.v = static_cast<const __half*>(v);
    p.q_stride = q_stride; p.k_stride = k_stride; p.v_stride = v_stride;
    p.q_weight = static_cast<const __half*>(q_norm_weight); p.k_weight = static_cast<const __half*>(k_norm_weight);
    p.cos_sin = cos_sin; p.positions = positions;
    p.lam_q = static_cast<const __half*>(lam_q); p.lam_k = static_cast<const __half*>(lam_k);
    p.q_out = static_cast<__half*>(q_out); p.k_out = static_cast<__half*>(k_out);
    p.kq = kq; p.ks = static_cast<const __half*>(ks); p.vq = vq; p.vs = static_cast<__half*>(vs); p.slots = slots;
    p.tokens = tokens; p.hq = hq; p.hkv = hkv; p.v_group = v_group > 0 ? v_group : d; p.num_slots = num_slots; p.eps = eps;
    const int64_t warps = int64_t(tokens) * (hq + hkv);
    const int blocks = int(cdiv64(warps, 4));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (d == 128) return launch_pdl(pre_attention_kernel<128>, dim3(blocks), dim3(128), 0, st, 1, p);
    return launch_pdl(pre_attention_kernel<64>, dim3(blocks), dim3(128), 0, st, 1, p);
}

int lq2_stage_decode(const int32_t* packed, int64_t* input_ids, int64_t* positions, int32_t* slot_mapping,
                     int32_t* context_lens, int32_t* block_tables, int batch, int rows_cap, int width,
                     int width_cap, void* stream) {
    if (!packed || !input_ids || !positions || !slot_mapping || !context_lens || !block_tables) return LQ2_ERR_ARG;
    if (batch < 0 || rows_cap <= 0 || batch > rows_cap || width < 0 || width_cap <= 0 || width > width_cap)
        return LQ2_ERR_SHAPE;
    const int64_t total = std::max<int64_t>(rows_cap, int64_t(rows_cap) * width_cap);
    return launch_pdl(stage_decode_kernel, dim3(unsigned(cdiv64(total, 256))), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), 1, packed, input_ids, positions, slot_mapping, context_lens,
                      block_tables, batch, rows_cap, width, width_cap);
}

}  // extern "C"
