// KV4 quantized write and prefix restore.
//
// kv4_store: replaces store_kv_quant (qslab/kernels/kv4/store.py:9-68).
// kv4_materialize: replaces materialize_kv (qslab/kernels/kv4/layout.py:9-47).
//
// Both are one-thread-per-word kernels: a pool word holds 8 consecutive
// channels of one (slot, head) as offset-binary nibbles, channel 8w + r in bits
// 4r..4r+3 (store.py:38-41).  The arithmetic is written so that the bytes match
// an IEEE fp32 evaluation of the reference's expressions exactly:
//   code = floor(min(max(x / s, -8), 7) + 0.5)          (store.py:37,49)
//   s_v  = max(amax_group(|v|) / 7, 1e-4), kept as fp32 for the codes and
//          stored as fp16                                (store.py:48-55)
//   restore = fp16(fp32(nibble - 8) * fp32(scale))       (layout.py:22-31)
#include "common.cuh"

namespace lq2 {

namespace {

__device__ __forceinline__ void unpack8(uint4 raw, float (&f)[8]) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 v = __half22float2(h[i]);
        f[2 * i] = v.x;
        f[2 * i + 1] = v.y;
    }
}

template <bool VEC>
__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
    if (VEC) {
        unpack8(*reinterpret_cast<const uint4*>(p), f);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = __half2float(p[i]);
    }
}
// fp32 keys / values: the reference's kernel converts whatever it loads to fp32
// (store.py:31,45), so fp32 inputs are quantized from their full precision
template <bool VEC>
__device__ __forceinline__ void load8(const float* p, float (&f)[8]) {
    if (VEC) {
        const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = p[i];
    }
}

__device__ __forceinline__ uint32_t encode(float x, float s) {
    const float q = floorf(fminf(fmaxf(__fdiv_rn(x, s), -8.0f), 7.0f) + 0.5f);
    return uint32_t(int(q) + 8) & 15u;
}

template <bool VEC, typename T>
__global__ void __launch_bounds__(256) kv4_store_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int64_t k_stride, int64_t v_stride,
    uint32_t* __restrict__ kq, const __half* __restrict__ ks, uint32_t* __restrict__ vq,
    __half* __restrict__ vs, const int32_t* __restrict__ slots, int tokens, int hkv, int nw,
    int words_per_group, int64_t num_slots) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int per_token = hkv * nw;
    const bool active = id < int64_t(tokens) * per_token;
    const int token = active ? int(id / per_token) : 0;
    const int rem = active ? int(id % per_token) : 0;
    const int h = rem / nw, w = rem % nw;
    const int d = nw * 8;

    float kf[8], sf[8], vf[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) { kf[i] = 0.f; sf[i] = 1.f; vf[i] = 0.f; }
    int64_t slot = -1;
    if (active) {
        slot = slots[token];
        load8<VEC>(k + int64_t(token) * k_stride + h * d + w * 8, kf);
        load8<VEC>(v + int64_t(token) * v_stride + h * d + w * 8, vf);
        load8<true>(ks + h * d + w * 8, sf);
    }
    const bool write = active && slot >= 0 && slot < num_slots;

    uint32_t kword = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) kword |= encode(kf[i], sf[i]) << (4 * i);

    // V: amax over the group's words.  Groups are aligned runs of
    // words_per_group lanes (a power of two <= 32), so a butterfly inside the
    // warp covers exactly one group; every lane of the warp takes part.
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(vf[i]));
    for (int off = 1; off < words_per_group; off <<= 1)
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float s_v = fmaxf(__fdiv_rn(amax, 7.0f), 1e-4f);
    uint32_t vword = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) vword |= encode(vf[i], s_v) << (4 * i);

    if (write) {
        const int64_t base = (slot * hkv + h) * nw + w;
        kq[base] = kword;
        vq[base] = vword;
        if (w % words_per_group == 0)
            vs[(slot * hkv + h) * (nw / words_per_group) + w / words_per_group] = __float2half_rn(s_v);
    }
}

__global__ void __launch_bounds__(256) kv4_materialize_kernel(
    const uint32_t* __restrict__ kq, const __half* __restrict__ ks, const uint32_t* __restrict__ vq,
    const __half* __restrict__ vs, const int64_t* __restrict__ slots, __half* __restrict__ k_out,
    __half* __restrict__ v_out, int tokens, int hkv, int nw, int words_per_group, int64_t num_slots) {
    pdl_launch_dependents();
    pdl_wait();
    const int64_t id = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int per_token = hkv * nw;
    if (id >= int64_t(tokens) * per_token) return;
    const int token = int(id / per_token), rem = int(id % per_token);
    const int h = rem / nw, w = rem % nw;
    const int d = nw * 8;
    const int64_t slot = slots[token];
    uint4 ko = make_uint4(0, 0, 0, 0), vo = make_uint4(0, 0, 0, 0);
    if (slot >= 0 && slot < num_slots) {
        const int64_t base = (slot * hkv + h) * nw + w;
        const uint32_t kw = kq[base], vw = vq[base];
        float sf[8];
        load8<true>(ks + h * d + w * 8, sf);
        const float s_v = __half2float(vs[(slot * hkv + h) * (nw / words_per_group) + w / words_per_group]);
        __half kh[8], vh[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float kc = float(int((kw >> (4 * i)) & 15u) - 8);
            const float vc = float(int((vw >> (4 * i)) & 15u) - 8);
            kh[i] = __float2half_rn(__fmul_rn(kc, sf[i]));
            vh[i] = __float2half_rn(__fmul_rn(vc, s_v));
        }
        ko = *reinterpret_cast<uint4*>(kh);
        vo = *reinterpret_cast<uint4*>(vh);
    }
    *reinterpret_cast<uint4*>(k_out + id * 8) = ko;
    *reinterpret_cast<uint4*>(v_out + id * 8) = vo;
}

}  // namespace

template <typename T>
static int store_launch(const T* k, const T* v, int64_t k_stride, int64_t v_stride, uint32_t* kq,
                        const __half* ks, uint32_t* vq, __half* vs, const int32_t* slots, int tokens,
                        int hkv, int d, int v_group, int64_t num_slots, cudaStream_t st) {
    const int nw = d / 8, wpg = v_group / 8;
    const int64_t total = int64_t(tokens) * hkv * nw;
    const int blocks = int(cdiv64(total, 256));
    constexpr int kVecElems = 16 / int(sizeof(T));       // elements per 16-byte access
    const bool vec = aligned(k, 16) && aligned(v, 16) && k_stride % kVecElems == 0 && v_stride % kVecElems == 0;
    if (vec)
        return launch_pdl(kv4_store_kernel<true, T>, dim3(blocks), dim3(256), 0, st, 1, k, v, k_stride, v_stride, kq,
                          ks, vq, vs, slots, tokens, hkv, nw, wpg, num_slots);
    return launch_pdl(kv4_store_kernel<false, T>, dim3(blocks), dim3(256), 0, st, 1, k, v, k_stride, v_stride, kq, ks,
                      vq, vs, slots, tokens, hkv, nw, wpg, num_slots);
}

int kv4_store_launch(const __half* k, const __half* v, int64_t k_stride, int64_t v_stride, uint32_t* kq,
                     const __half* ks, uint32_t* vq, __half* vs, const int32_t* slots, int tokens,
                     int hkv, int d, int v_group, int64_t num_slots, cudaStream_t st) {
    return store_launch(k, v, k_stride, v_stride, kq, ks, vq, vs, slots, tokens, hkv, d, v_group, num_slots, st);
}

int kv4_store_f32_launch(const float* k, const float* v, int64_t k_stride, int64_t v_stride, uint32_t* kq,
                         const __half* ks, uint32_t* vq, __half* vs, const int32_t* slots, int tokens,
                         int hkv, int d, int v_group, int64_t num_slots, cudaStream_t st) {
    return store_launch(k, v, k_stride, v_stride, kq, ks, vq, vs, slots, tokens, hkv, d, v_group, num_slots, st);
}

int kv4_materialize_launch(const uint32_t* kq, const __half* ks, const uint32_t* vq, const __half* vs,
                           const int64_t* slots, __half* k_out, __half* v_out, int tokens, int hkv,
                           int d, int v_group, int64_t num_slots, cudaStream_t st) {
    const int nw = d / 8, wpg = v_group / 8;
    const int64_t total = int64_t(tokens) * hkv * nw;
    const int blocks = int(cdiv64(total, 256));
    return launch_pdl(kv4_materialize_kernel, dim3(blocks), dim3(256), 0, st, 1, kq, ks, vq, vs, slots, k_out, v_out,
                      tokens, hkv, nw, wpg, num_slots);
}

}  // namespace lq2
