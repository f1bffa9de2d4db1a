// Paged attention over the int4 KV pool: decode (one query position) and
// multi-position verify, split-KV flash-decoding with an online softmax.
//
// Replaces paged_attention_decode and its three Triton kernels
// (qslab/kernels/kv4/paged_attention.py:11-150: decode kernel, split merge and
// launcher; qslab/kernels/kv4/grouped_attention.py:7-63: grouped verify).
//
// Three kernels share the launcher at the end of this file:
//   kv4_decode_fast_kernel  at most 8 query rows per KV head (decode, D 64 or 128): per-warp cp.async
//                           rings, the cache as the 16-row MMA operand, codes as fp16 subnormals;
//   kv4_verify_kernel       17..64 query rows per KV head at D = 128 (16-position verify, and the
//                           prefix part of chunked prefill): the tile dequantised once per CTA into
//                           shared memory, ldmatrix operands;
//   kv4_attention_kernel    every other geometry: one CTA per (sequence, KV head, split), query rows
//                           row = m * rep + head_in_group cut into tiles of 16, warp w on row tile
//                           w % RT and on every (4/RT)-th 16-token block, operands unpacked in registers.
// In all of them every query head of a GQA group - and for verify all M positions - shares a single
// read of the packed K/V bytes, both products run on the warp-level tensor-core op m16n8k16 with fp32
// accumulation, and scores, running maximum, denominator and O stay fp32:
//   S = Q' K^T : Q' = q * ks carries the static per-channel K scale, so K enters as exact integers;
//                Q' is exact in fp32 and is split into a high and a low fp16 part (one rounded fp16
//                would shift all scores of a row by the same channel-wise error);
//   O += P' V  : P' = p * vs carries the V scale of the token and group, V enters as exact integers
//                (the generic kernel dequantises V to fp16 (nibble - 8) * vs instead, as the
//                reference's verify kernel does, grouped_attention.py:50-53).
//
// Splits.  The split count depends on shapes only.  Each CTA writes an fp32
// partial (O, max, denominator) per row, takes a ticket, and the last CTA of a
// (sequence, KV head) merges the partials in split order (merge_splits) and writes fp16.
#include <math.h>

#include <mutex>

#include "common.cuh"

// Built-in scratch for lq2_kv4_attention_static: callers that cannot allocate
// device memory get the split partials and ticket counters from this array
// instead of a workspace argument.  Every device that loads the library holds
// these 16 MiB until the process exits.  In host code the symbol below is only a
// handle; its device address is resolved per device with cudaGetSymbolAddress.
#define LQ2_BUILTIN_SCRATCH_BYTES (size_t(16) << 20)
static __device__ __align__(256) unsigned char g_lq2_attention_scratch[LQ2_BUILTIN_SCRATCH_BYTES];

namespace lq2 {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTile = 16;  // tokens per MMA block

struct AttnParams {
    const __half* q;
    int64_t q_stride;
    const uint32_t* kq;
    const __half* ks;
    const uint32_t* vq;
    const __half* vs;
    const int32_t* bt;
    const int32_t* lens;
    __half* out;
    int batch, m, hq, hkv, page, max_blocks, ng, vg_shift;
    int num_blocks;
    int page_shift;    // log2(page) when page is a power of two, else -1
    int splits;
    float sl2;  // D^-0.5 * log2(e)
    float* partial;
    int* counters;
    // Row m of a sequence reads positions [0, len + m * pos_step): 1 for decode / verify (causal over the
    // drafts), 0 when all rows of a block attend to the same cached prefix (chunked prefill).
    int pos_step;
    float* lse;        // optional [batch * m, hq]: natural-log sum of exp(scores) per row, -inf without keys
};

__device__ __forceinline__ float lse_of(float max2, float den) {     // from the base-2 running maximum
    return den > 0.f ? (max2 + log2f(den)) * 0.6931471805599453f : -INFINITY;
}

template <int D>
struct KWords;
template <>
struct KWords<128> { using type = uint4; };
template <>
struct KWords<64> { using type = uint2; };

template <int D>
struct VWords;
template <>
struct VWords<128> { using type = uint2; };
template <>
struct VWords<64> { using type = uint32_t; };

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
__device__ __forceinline__ uint32_t word_of(const uint2& v, int i) { return i == 0 ? v.x : v.y; }
__device__ __forceinline__ uint32_t word_of(const uint32_t& v, int) { return v; }

__device__ __forceinline__ void ldg(uint4& d, const uint32_t* p) { d = ldg_stream_u4(p); }
__device__ __forceinline__ void ldg(uint2& d, const uint32_t* p) { d = ldg_stream_u2(p); }
__device__ __forceinline__ void ldg(uint32_t& d, const uint32_t* p) { d = ldg_stream_u1(p); }

__device__ __forceinline__ uint32_t pack_h2(float a, float b) { return h2_as_u32(__floats2half2_rn(a, b)); }
// 2^x for x <= 0 (or -inf): the hardware approximation, 2 ulp
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
    return y;
}

// A split's partial: per row D sums, then (running max in the base-2 domain, denominator), padded to
// D + 4 floats so that rows are 16-byte aligned.
__host__ __device__ constexpr int part_row(int d) { return d + 4; }

// Merge of the split partials by the last CTA of a (sequence, head group).  `units` heads x `rows` rows;
// part_of(u) is the base of unit u's [splits][rows][D + 4] partials.  The (max, denominator) pairs are
// first brought to shared memory in one sweep - read on demand they would put two dependent memory round
// trips per split on every thread's path - and the sums are then read four splits at a time with
// independent 16-byte loads.  A split that saw no token wrote (-inf, 0) and possibly no sums: its sums are
// never used.  sm_stat needs units * splits * rows entries.
template <int D, int THREADS, typename PartOf, typename Store>
__device__ __forceinline__ void merge_splits(int units, int rows, int splits, float2* sm_stat, PartOf part_of,
                                             Store store) {
    constexpr int RS = part_row(D), V = D / 4;
    const int tid = threadIdx.x;
    const int per_unit = splits * rows;
    for (int i = tid; i < units * per_unit; i += THREADS) {
        const int u = i / per_unit, r = i - u * per_unit;                 // r = split * rows + row
        sm_stat[i] = __ldcg(reinterpret_cast<const float2*>(part_of(u) + int64_t(r) * RS + D));
    }
    __syncthreads();
    for (int e = tid; e < units * rows * V; e += THREADS) {
        const int d = (e % V) * 4, ur = e / V, u = ur / rows, row = ur - u * rows;
        const float2* st = sm_stat + u * per_unit + row;
        float mx = -INFINITY;
        for (int sp = 0; sp < splits; ++sp) mx = fmaxf(mx, st[sp * rows].x);
        const float safe = mx == -INFINITY ? 0.f : mx;
        const float* src = part_of(u) + int64_t(row) * RS + d;
        const int64_t step = int64_t(rows) * RS;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float den = 0.f;
        auto add = [&](const float4& v, const float2& s2) {
            if (s2.x != -INFINITY) {
                const float f = ex2(s2.x - safe);
                acc.x += v.x * f; acc.y += v.y * f; acc.z += v.z * f; acc.w += v.w * f;
                den += s2.y * f;
            }
        };
        int sp = 0;
        for (; sp + 4 <= splits; sp += 4) {
            float4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = __ldcg(reinterpret_cast<const float4*>(src + (sp + k) * step));
#pragma unroll
            for (int k = 0; k < 4; ++k) add(v[k], st[(sp + k) * rows]);
        }
        for (; sp < splits; ++sp) add(__ldcg(reinterpret_cast<const float4*>(src + sp * step)), st[sp * rows]);
        store(u, row, d, acc, 1.f / fmaxf(den, 1e-20f), lse_of(safe, den));
    }
}

__device__ __forceinline__ void store_h4(__half* dst, const float4& a, float inv) {
    const __half2 h01 = __floats2half2_rn(a.x * inv, a.y * inv), h23 = __floats2half2_rn(a.z * inv, a.w * inv);
    *reinterpret_cast<uint2*>(dst) = make_uint2(h2_as_u32(h01), h2_as_u32(h23));
}

// RT: 16-row query tiles per (sequence, KV head): ceil(M * rep / 16), 3 rounded up to 4.
template <int D, int RT>
__global__ void __launch_bounds__(kThreads) kv4_attention_kernel(const AttnParams p) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int NW = D / 8;          // words per (token, head)
    constexpr int KWT = NW / 4;        // K words per lane per token (lanes t = 0..3 split the row)
    constexpr int VWT = NW / 8;        // V words per lane per token (lanes g = 0..7 split the row)
    constexpr int NT = 8 * VWT;        // n-tiles (of 8 channels) of the PV product per lane
    constexpr int WT = kWarps / RT;    // warps that split the tokens of one row tile
    constexpr int ROWS = 16 * RT;
    using KW = typename KWords<D>::type;
    using VW = typename VWords<D>::type;

    __shared__ __align__(16) float sm_raw[kWarps * 16 * 128];       // 32 KB: per-warp sums, later the merge's pairs
    float (*sm_o)[16][D] = reinterpret_cast<float (*)[16][D]>(sm_raw);
    __shared__ float sm_m[kWarps][16];
    __shared__ float sm_l[kWarps][16];
    __shared__ int s_ticket;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int rt = warp % RT, ws = warp / RT;
    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int rep = p.hq / p.hkv;
    const int rows_valid = p.m * rep;

    const int capacity = p.max_blocks * p.page;
    const int len = p.lens[seq];
    const int reach = min(len + (p.m - 1) * p.pos_step, capacity);   // keys any row of this sequence reads
    const int tiles = reach > 0 ? (reach + kTile - 1) / kTile : 0;
    const int per_split = (tiles + p.splits - 1) / p.splits;
    const int tile_begin = split * per_split;
    const int tile_end = min(tiles, tile_begin + per_split);

    // ---- Q' fragments: rows r_lo = 16*rt + g and r_hi = r_lo + 8
    const int r_lo = 16 * rt + g, r_hi = r_lo + 8;
    const bool v_lo = r_lo < rows_valid, v_hi = r_hi < rows_valid;
    const int m_lo = v_lo ? r_lo / rep : 0, m_hi = v_hi ? r_hi / rep : 0;
    const int lim_lo = v_lo ? min(len + m_lo * p.pos_step, capacity) : 0;
    const int lim_hi = v_hi ? min(len + m_hi * p.pos_step, capacity) : 0;
    // Q' = q * ks is exact in fp32 and is carried as a high and a low fp16 part (two MMAs per operand):
    // rounded to one fp16 it would shift every score of a row by the same channel-wise error, which
    // does not average out over the tokens.
    uint32_t qa[KWT][2][4], ql[KWT][2][4];
    {
        const __half* q_lo = p.q + int64_t(seq * p.m + m_lo) * p.q_stride + (kvh * rep + (v_lo ? r_lo % rep : 0)) * D;
        const __half* q_hi = p.q + int64_t(seq * p.m + m_hi) * p.q_stride + (kvh * rep + (v_hi ? r_hi % rep : 0)) * D;
        const __half* ksp = p.ks + kvh * D;
#pragma unroll
        for (int wi = 0; wi < KWT; ++wi) {
            const int d0 = 8 * (t * KWT + wi);
            float lo[8], hi[8], lo2[8], hi2[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float sc = __half2float(ksp[d0 + i]);
                const float a = v_lo ? __half2float(q_lo[d0 + i]) * sc : 0.f;
                const float b = v_hi ? __half2float(q_hi[d0 + i]) * sc : 0.f;
                lo[i] = __half2float(__float2half_rn(a));
                hi[i] = __half2float(__float2half_rn(b));
                lo2[i] = a - lo[i];
                hi2[i] = b - hi[i];
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                qa[wi][h][0] = pack_h2(lo[2 * h], lo[2 * h + 4]);
                qa[wi][h][1] = pack_h2(hi[2 * h], hi[2 * h + 4]);
                qa[wi][h][2] = pack_h2(lo[2 * h + 1], lo[2 * h + 5]);
                qa[wi][h][3] = pack_h2(hi[2 * h + 1], hi[2 * h + 5]);
                ql[wi][h][0] = pack_h2(lo2[2 * h], lo2[2 * h + 4]);
                ql[wi][h][1] = pack_h2(hi2[2 * h], hi2[2 * h + 4]);
                ql[wi][h][2] = pack_h2(lo2[2 * h + 1], lo2[2 * h + 5]);
                ql[wi][h][3] = pack_h2(hi2[2 * h + 1], hi2[2 * h + 5]);
            }
        }
    }

    float o[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[j][c] = 0.f;
    float mx_lo = -INFINITY, mx_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

    const __half2 k1032 = __floats2half2_rn(1032.f, 1032.f);
    const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
    const __half2 km72 = __floats2half2_rn(-72.f, -72.f);
    const int vgrp = (8 * VWT * g) >> p.vg_shift;     // V scale group of this lane's channels

    KW kw[2], kwn[2];
    VW vw[4], vwn[4];
    __half vsc[4], vscn[4];
    bool live = false, live_n = false;

    auto fetch = [&](int tile, KW (&k_)[2], VW (&v_)[4], __half (&s_)[4], bool& ok) {
        const int pos0 = tile * kTile;
        const int raw = p.bt[int64_t(seq) * p.max_blocks + pos0 / p.page];
        ok = raw >= 0;
        if (!ok) return;
        const int blk = min(raw, p.num_blocks - 1);
        const int64_t slot0 = int64_t(blk) * p.page + pos0 % p.page;
#pragma unroll
        for (int n8 = 0; n8 < 2; ++n8)
            ldg(k_[n8], p.kq + ((slot0 + g + 8 * n8) * p.hkv + kvh) * NW + t * KWT);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t slot = slot0 + 2 * t + (i & 1) + 8 * (i >> 1);
            ldg(v_[i], p.vq + (slot * p.hkv + kvh) * NW + g * VWT);
            s_[i] = p.vs[(slot * p.hkv + kvh) * p.ng + vgrp];
        }
    };

    int tile = tile_begin + ws;
    if (tile < tile_end) fetch(tile, kw, vw, vsc, live);
    for (; tile < tile_end; tile += WT) {
        const int next = tile + WT;
        live_n = false;
        if (next < tile_end) fetch(next, kwn, vwn, vscn, live_n);
        if (live) {
            // ---- S = Q' K^T for 16 tokens (two n8 blocks)
            float s[2][4], sl[2][4];
#pragma unroll
            for (int n8 = 0; n8 < 2; ++n8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) s[n8][c] = sl[n8][c] = 0.f;
#pragma unroll
                for (int wi = 0; wi < KWT; ++wi) {
                    const uint32_t w = word_of(kw[n8], wi);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t x = w >> (8 * h);
                        const uint32_t b0 = h2_as_u32(__hsub2(u32_as_h2(and_or(x, 0x000f000fu, 0x64006400u)), k1032));
                        const uint32_t b1 = h2_as_u32(__hfma2(u32_as_h2(and_or(x, 0x00f000f0u, 0x64006400u)), k16th, km72));
                        mma_m16n8k16(s[n8], qa[wi][h][0], qa[wi][h][1], qa[wi][h][2], qa[wi][h][3], b0, b1);
                        mma_m16n8k16(sl[n8], ql[wi][h][0], ql[wi][h][1], ql[wi][h][2], ql[wi][h][3], b0, b1);
                    }
                }
            }
            // ---- mask, online softmax (base-2 domain)
            const int pos0 = tile * kTile;
            float t_lo = -INFINITY, t_hi = -INFINITY;
#pragma unroll
            for (int n8 = 0; n8 < 2; ++n8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const int pos = pos0 + 8 * n8 + 2 * t + (c & 1);
                    const int lim = c < 2 ? lim_lo : lim_hi;
                    const float v = pos < lim ? (s[n8][c] + sl[n8][c]) * p.sl2 : -INFINITY;
                    s[n8][c] = v;
                    if (c < 2) t_lo = fmaxf(t_lo, v); else t_hi = fmaxf(t_hi, v);
                }
            }
            t_lo = fmaxf(t_lo, __shfl_xor_sync(0xffffffffu, t_lo, 1));
            t_lo = fmaxf(t_lo, __shfl_xor_sync(0xffffffffu, t_lo, 2));
            t_hi = fmaxf(t_hi, __shfl_xor_sync(0xffffffffu, t_hi, 1));
            t_hi = fmaxf(t_hi, __shfl_xor_sync(0xffffffffu, t_hi, 2));
            const float n_lo = fmaxf(mx_lo, t_lo), n_hi = fmaxf(mx_hi, t_hi);
            const float safe_lo = n_lo == -INFINITY ? 0.f : n_lo;
            const float safe_hi = n_hi == -INFINITY ? 0.f : n_hi;
            const float a_lo = exp2f(mx_lo - safe_lo), a_hi = exp2f(mx_hi - safe_hi);
            mx_lo = n_lo;
            mx_hi = n_hi;
            float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
            for (int n8 = 0; n8 < 2; ++n8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float e = exp2f(s[n8][c] - (c < 2 ? safe_lo : safe_hi));
                    s[n8][c] = e;
                    if (c < 2) sum_lo += e; else sum_hi += e;
                }
            }
            l_lo = l_lo * a_lo + sum_lo;
            l_hi = l_hi * a_hi + sum_hi;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
                o[j][0] *= a_lo; o[j][1] *= a_lo;
                o[j][2] *= a_hi; o[j][3] *= a_hi;
            }
            const uint32_t pa0 = pack_h2(s[0][0], s[0][1]), pa1 = pack_h2(s[0][2], s[0][3]);
            const uint32_t pa2 = pack_h2(s[1][0], s[1][1]), pa3 = pack_h2(s[1][2], s[1][3]);
            // ---- O += P V.  Lane (g, t) supplies tokens 2t, 2t+1 (k-slots 2t, 2t+1) and
            // 2t+8, 2t+9 for channels 8*VWT*g + j, j = 0..NT-1.
            const __half2 sc_a = __halves2half2(vsc[0], vsc[1]);
            const __half2 sc_b = __halves2half2(vsc[2], vsc[3]);
#pragma unroll
            for (int wsel = 0; wsel < VWT; ++wsel) {
                const uint32_t wa0 = word_of(vw[0], wsel), wa1 = word_of(vw[1], wsel);
                const uint32_t wb0 = word_of(vw[2], wsel), wb1 = word_of(vw[3], wsel);
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint32_t sel = b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12);
                    const uint32_t xa = __byte_perm(wa0, wa1, sel);
                    const uint32_t xb = __byte_perm(wb0, wb1, sel);
                    const __half2 ea = __hsub2(u32_as_h2(and_or(xa, 0x000f000fu, 0x64006400u)), k1032);
                    const __half2 eb = __hsub2(u32_as_h2(and_or(xb, 0x000f000fu, 0x64006400u)), k1032);
                    mma_m16n8k16(o[8 * wsel + 2 * b], pa0, pa1, pa2, pa3,
                                 h2_as_u32(__hmul2(ea, sc_a)), h2_as_u32(__hmul2(eb, sc_b)));
                    const __half2 fa = __hfma2(u32_as_h2(and_or(xa, 0x00f000f0u, 0x64006400u)), k16th, km72);
                    const __half2 fb = __hfma2(u32_as_h2(and_or(xb, 0x00f000f0u, 0x64006400u)), k16th, km72);
                    mma_m16n8k16(o[8 * wsel + 2 * b + 1], pa0, pa1, pa2, pa3,
                                 h2_as_u32(__hmul2(fa, sc_a)), h2_as_u32(__hmul2(fb, sc_b)));
                }
            }
        }
        live = live_n;
#pragma unroll
        for (int i = 0; i < 2; ++i) kw[i] = kwn[i];
#pragma unroll
        for (int i = 0; i < 4; ++i) { vw[i] = vwn[i]; vsc[i] = vscn[i]; }
    }

    // ---- per-warp state to shared memory.  o[j][0] is (row r_lo, channel 8*VWT*(2t) + j),
    // o[j][1] channel 8*VWT*(2t+1) + j; o[j][2..3] the same for r_hi.
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
#pragma unroll
    for (int j = 0; j < NT; ++j) {
        sm_o[warp][g][NT * (2 * t) + j] = o[j][0];
        sm_o[warp][g][NT * (2 * t + 1) + j] = o[j][1];
        sm_o[warp][g + 8][NT * (2 * t) + j] = o[j][2];
        sm_o[warp][g + 8][NT * (2 * t + 1) + j] = o[j][3];
    }
    if (t == 0) {
        sm_m[warp][g] = mx_lo; sm_m[warp][g + 8] = mx_hi;
        sm_l[warp][g] = l_lo;  sm_l[warp][g + 8] = l_hi;
    }
    __syncthreads();

    // ---- merge the WT warps of each row tile; write the result or this split's partial
    const int splits = p.splits;
    float* part = p.partial + (int64_t(seq * p.hkv + kvh) * splits) * rows_valid * part_row(D);
    for (int e = tid; e < ROWS * D; e += kThreads) {
        const int row = e / D, d = e % D;
        if (row >= rows_valid) continue;
        const int tl = row / 16, r16 = row % 16;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < WT; ++w) mx = fmaxf(mx, sm_m[w * RT + tl][r16]);
        const float safe = mx == -INFINITY ? 0.f : mx;
        float acc = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < WT; ++w) {
            const float f = exp2f(sm_m[w * RT + tl][r16] - safe);
            acc += sm_o[w * RT + tl][r16][d] * f;
            den += sm_l[w * RT + tl][r16] * f;
        }
        if (splits == 1) {
            const int mrow = row / rep, head = kvh * rep + row % rep;
            p.out[(int64_t(seq * p.m + mrow) * p.hq + head) * D + d] = __float2half_rn(acc / fmaxf(den, 1e-20f));
            if (d == 0 && p.lse) p.lse[int64_t(seq * p.m + mrow) * p.hq + head] = lse_of(safe, den);
        } else {
            float* dst = part + (int64_t(split) * rows_valid + row) * part_row(D);
            __stcg(dst + d, acc);
            if (d == 0) { __stcg(dst + D, mx); __stcg(dst + D + 1, den); }
        }
    }
    if (splits == 1) return;

    __threadfence();
    __syncthreads();
    int* counter = p.counters + seq * p.hkv + kvh;
    if (tid == 0) s_ticket = atomicAdd(counter, 1);
    __syncthreads();
    if (s_ticket != splits - 1) return;
    __threadfence();
    merge_splits<D, kThreads>(
        1, rows_valid, splits, reinterpret_cast<float2*>(sm_raw), [&](int) { return part; },
        [&](int, int row, int d, const float4& acc, float inv, float lse) {
            store_h4(p.out + (int64_t(seq * p.m + row / rep) * p.hq + kvh * rep + row % rep) * D + d, acc, inv);
            if (d == 0 && p.lse) p.lse[int64_t(seq * p.m + row / rep) * p.hq + kvh * rep + row % rep] = lse;
        });
    if (tid == 0) *counter = 0;
}

// =====================================================================================
// Verify path: 17..64 query rows per KV head (M draft positions x the GQA group), D = 128.
//
// Replaces kv4_grouped_verify_kernel (qslab/kernels/kv4/grouped_attention.py:7-63), which
// dequantises every K/V tile once per 16-row query block.  Here the CTA of one (sequence, KV
// head, split) dequantises each 32-token tile ONCE, cooperatively, into shared memory as
// the exact fp16 integers (nibble - 8), and every warp (one 16-row query tile each) reads its
// MMA operands from there with ldmatrix.  The V scales (per token and group) multiply the
// probabilities instead, P' = p * vs, so the codes stay exact.
// The static K scale is folded into the queries, Q' = q * ks, which is exact in fp32 and is
// kept in shared memory as a high and a low fp16 part (S = Q'hi K^T + Q'lo K^T): rounded to one
// fp16 it would shift every score of a row by the same channel-wise error, and rounding
// K * ks instead costs as much.
// The packed words of the next two tiles are in flight (two register sets) while the current
// tile is multiplied; the two fp16 buffers alternate, so there is one CTA barrier per tile.
// Within every 8 channels the tiles keep the order the nibble masks produce, (0,4,1,5,2,6,3,7);
// Q' is stored in the same order and O is put back in natural order at the write-out.
// =====================================================================================
constexpr int kVTile = 32;                 // tokens per tile
constexpr int kVStride = 128 + 8;          // halves per row: +16 bytes keep ldmatrix conflict-free
constexpr int kVTileHalves = kVTile * kVStride;

template <int RT>
struct VerifyLayout {
    static constexpr int Q_HALVES = 16 * RT * kVStride;                 // one of the two parts of Q'
    static constexpr int SMEM_BYTES = (2 * Q_HALVES + 4 * kVTileHalves) * 2;
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem_row) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* smem_row) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem_row));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}

template <int RT>
__global__ void __launch_bounds__(kThreads, 3) kv4_verify_kernel(const AttnParams p) {
    pdl_launch_dependents();
    pdl_wait();
    constexpr int D = 128, NW = 16, ROWS = 16 * RT;
    extern __shared__ __align__(16) unsigned char vsm[];
    __half* sm_qh = reinterpret_cast<__half*>(vsm);
    __half* sm_ql = sm_qh + VerifyLayout<RT>::Q_HALVES;
    __half* sm_k = sm_ql + VerifyLayout<RT>::Q_HALVES;      // [2][kVTileHalves]
    __half* sm_v = sm_k + 2 * kVTileHalves;                 // [2][kVTileHalves]
    __shared__ uint32_t sm_vs[2][kVTile];                   // V scales of the tile: (group 0, group 1) per token
    __shared__ int s_ticket;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int split = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
    const int rep = p.hq / p.hkv;
    const int rows_valid = p.m * rep;

    const int capacity = p.max_blocks * p.page;
    const int len = p.lens[seq];
    const int reach = min(len + (p.m - 1) * p.pos_step, capacity);
    const int tiles = reach > 0 ? (reach + kVTile - 1) / kVTile : 0;
    const int per_split = (tiles + p.splits - 1) / p.splits;
    const int tile_begin = split * per_split;
    const int tile_end = min(tiles, tile_begin + per_split);

    const int splits = p.splits;
    float* part = p.partial + (int64_t(seq * p.hkv + kvh) * splits) * rows_valid * part_row(D);
    const bool idle = tile_begin >= tile_end;               // block-uniform: a split beyond this sequence's end
    if (idle && splits > 1) {                               // only its (max, denominator) = (-inf, 0) is recorded
        for (int row = tid; row < rows_valid; row += kThreads) {
            float* dst = part + (int64_t(split) * rows_valid + row) * part_row(D);
            __stcg(dst + D, -INFINITY);
            __stcg(dst + D + 1, 0.f);
        }
    }

    const bool mma_warp = warp < RT;
    const int r_lo = 16 * warp + g, r_hi = r_lo + 8;
    const bool v_lo = mma_warp && r_lo < rows_valid, v_hi = mma_warp && r_hi < rows_valid;
    const int lim_lo = v_lo ? min(len + r_lo / rep * p.pos_step, capacity) : 0;
    const int lim_hi = v_hi ? min(len + r_hi / rep * p.pos_step, capacity) : 0;
    int lim_min = min(lim_lo, lim_hi);                        // tiles wholly below it need no mask
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) lim_min = min(lim_min, __shfl_xor_sync(0xffffffffu, lim_min, off));

    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[j][c] = 0.f;
    float mx_lo = -INFINITY, mx_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

    // lane-constant operand addresses
    const __half* a_hi = sm_qh + (16 * warp + (lane & 7) + 8 * ((lane >> 3) & 1)) * kVStride + 8 * (lane >> 4);
    const __half* a_lo = a_hi + VerifyLayout<RT>::Q_HALVES;
    const int kb_off = (lane & 7) * kVStride + (lane >> 3) * 8;
    const int vb_off = (8 * ((lane >> 3) & 1) + (lane & 7)) * kVStride + (lane >> 4) * 8;

    // ---- cooperative dequantisation: thread (token = tid / 4, quarter = tid % 4) owns 4 K and 4 V words
    const int dq_tok = tid >> 2, dq_q = tid & 3;
    const int dq_off = dq_tok * kVStride + 32 * dq_q;
    const __half2 k1032 = __floats2half2_rn(1032.f, 1032.f);
    const __half2 k16th = __floats2half2_rn(0.0625f, 0.0625f);
    const __half2 km72 = __floats2half2_rn(-72.f, -72.f);
    const int64_t row_words = int64_t(p.hkv) * NW;
    const int64_t lane_words = dq_tok * row_words + kvh * NW + 4 * dq_q;
    uint4 kw[2], vw[2];
    uint32_t vsc[2] = {0u, 0u};
    bool live[2] = {false, false};
    int raw_ahead = -1;

    // The block-table entry of a tile decides whether the tile is fetched at all, so waiting for it would
    // stall the warp for a memory round trip per tile: it is read one step before it is used.
    const int32_t* bt_row = p.bt + int64_t(seq) * p.max_blocks;
    auto table_entry = [&](int tile) { return tile < tile_end ? bt_row[tile * kVTile / p.page] : -1; };
    auto fetch = [&](int tile, int raw, uint4& kw_, uint4& vw_, uint32_t& vsc_, bool& live_) {
        live_ = tile < tile_end && raw >= 0;                      // a tile never straddles pages (page % 32 == 0)
        if (!live_) return;
        const int pos0 = tile * kVTile;
        const int64_t slot0 = int64_t(min(raw, p.num_blocks - 1)) * p.page + pos0 % p.page;
        kw_ = ldg_stream_u4(p.kq + slot0 * row_words + lane_words);
        vw_ = ldg_stream_u4(p.vq + slot0 * row_words + lane_words);
        if (dq_q == 0) {                                          // one lane per token fetches its scales
            const __half* sp = p.vs + ((slot0 + dq_tok) * p.hkv + kvh) * p.ng;
            vsc_ = p.ng == 2 ? *reinterpret_cast<const uint32_t*>(sp) : h2_as_u32(__half2half2(sp[0]));
        }
    };
    auto convert = [&](int buf, const uint4& kw_, const uint4& vw_, uint32_t vsc_) {   // registers -> fp16 rows
        const uint32_t kws[4] = {kw_.x, kw_.y, kw_.z, kw_.w}, vws[4] = {vw_.x, vw_.y, vw_.z, vw_.w};
        if (dq_q == 0) sm_vs[buf][dq_tok] = vsc_;
        __half* kdst = sm_k + buf * kVTileHalves + dq_off;
        __half* vdst = sm_v + buf * kVTileHalves + dq_off;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t a = kws[i], a8 = a >> 8, b = vws[i], b8 = b >> 8;
            uint4 ko, vo;
            // (n0,n4) (n1,n5) (n2,n6) (n3,n7) as exact integers (nibble - 8)
            ko.x = h2_as_u32(__hsub2(u32_as_h2(and_or(a, 0x000f000fu, 0x64006400u)), k1032));
            ko.y = h2_as_u32(__hfma2(u32_as_h2(and_or(a, 0x00f000f0u, 0x64006400u)), k16th, km72));
            ko.z = h2_as_u32(__hsub2(u32_as_h2(and_or(a8, 0x000f000fu, 0x64006400u)), k1032));
            ko.w = h2_as_u32(__hfma2(u32_as_h2(and_or(a8, 0x00f000f0u, 0x64006400u)), k16th, km72));
            vo.x = h2_as_u32(__hsub2(u32_as_h2(and_or(b, 0x000f000fu, 0x64006400u)), k1032));
            vo.y = h2_as_u32(__hfma2(u32_as_h2(and_or(b, 0x00f000f0u, 0x64006400u)), k16th, km72));
            vo.z = h2_as_u32(__hsub2(u32_as_h2(and_or(b8, 0x000f000fu, 0x64006400u)), k1032));
            vo.w = h2_as_u32(__hfma2(u32_as_h2(and_or(b8, 0x00f000f0u, 0x64006400u)), k16th, km72));
            *reinterpret_cast<uint4*>(kdst + 8 * i) = ko;
            *reinterpret_cast<uint4*>(vdst + 8 * i) = vo;
        }
    };

    // One tile: `par` is the parity of (tile - tile_begin): the fp16 buffer it reads and the register set
    // the tile after next is fetched into.
    auto step = [&](auto PAR, int tile) {
        constexpr int par = decltype(PAR)::value;
        const bool cur_live = live[par];
        const int raw_now = raw_ahead;
        raw_ahead = table_entry(tile + 3);
        fetch(tile + 2, raw_now, kw[par], vw[par], vsc[par], live[par]);   // this set was converted one step ago
        if (cur_live && mma_warp) {
            const __half* kb = sm_k + par * kVTileHalves + kb_off;
            const __half* vb = sm_v + par * kVTileHalves + vb_off;
            // ---- S = Q' K^T: 16 rows x 32 tokens, high and low parts in separate accumulators
            float s[4][4], sl[4][4];
#pragma unroll
            for (int n8 = 0; n8 < 4; ++n8)
#pragma unroll
                for (int c = 0; c < 4; ++c) s[n8][c] = sl[n8][c] = 0.f;
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {                      // 32 channels = two k-chunks per step
                uint32_t ah0[4], ah1[4], al0[4], al1[4];
                ldsm_x4(ah0, a_hi + 32 * q4);
                ldsm_x4(ah1, a_hi + 32 * q4 + 16);
                ldsm_x4(al0, a_lo + 32 * q4);
                ldsm_x4(al1, a_lo + 32 * q4 + 16);
#pragma unroll
                for (int n8 = 0; n8 < 4; ++n8) {
                    uint32_t bf[4];
                    ldsm_x4(bf, kb + 8 * n8 * kVStride + 32 * q4);
                    mma_m16n8k16(s[n8], ah0[0], ah0[1], ah0[2], ah0[3], bf[0], bf[1]);
                    mma_m16n8k16(sl[n8], al0[0], al0[1], al0[2], al0[3], bf[0], bf[1]);
                    mma_m16n8k16(s[n8], ah1[0], ah1[1], ah1[2], ah1[3], bf[2], bf[3]);
                    mma_m16n8k16(sl[n8], al1[0], al1[1], al1[2], al1[3], bf[2], bf[3]);
                }
            }
            // ---- mask (last tiles only), online softmax in the base-2 domain
            const int pos0 = tile * kVTile;
            const bool masked = pos0 + kVTile > lim_min;          // warp-uniform
            float t_lo = -INFINITY, t_hi = -INFINITY;
#pragma unroll
            for (int n8 = 0; n8 < 4; ++n8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float v = s[n8][c] + sl[n8][c];
                    if (masked) {
                        const int pos = pos0 + 8 * n8 + 2 * t + (c & 1);
                        if (pos >= (c < 2 ? lim_lo : lim_hi)) v = -INFINITY;
                    }
                    s[n8][c] = v;
                    if (c < 2) t_lo = fmaxf(t_lo, v); else t_hi = fmaxf(t_hi, v);
                }
            }
            t_lo = fmaxf(t_lo, __shfl_xor_sync(0xffffffffu, t_lo, 1));
            t_lo = fmaxf(t_lo, __shfl_xor_sync(0xffffffffu, t_lo, 2));
            t_hi = fmaxf(t_hi, __shfl_xor_sync(0xffffffffu, t_hi, 1));
            t_hi = fmaxf(t_hi, __shfl_xor_sync(0xffffffffu, t_hi, 2));
            const float n_lo = fmaxf(mx_lo, t_lo * p.sl2), n_hi = fmaxf(mx_hi, t_hi * p.sl2);   // sl2 > 0
            const float safe_lo = n_lo == -INFINITY ? 0.f : n_lo;
            const float safe_hi = n_hi == -INFINITY ? 0.f : n_hi;
            const float f_lo = ex2(mx_lo - safe_lo), f_hi = ex2(mx_hi - safe_hi);
            mx_lo = n_lo;
            mx_hi = n_hi;
            float sum_lo = 0.f, sum_hi = 0.f;
#pragma unroll
            for (int n8 = 0; n8 < 4; ++n8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const float e = ex2(fmaf(s[n8][c], p.sl2, c < 2 ? -safe_lo : -safe_hi));
                    s[n8][c] = e;
                    if (c < 2) sum_lo += e; else sum_hi += e;
                }
            }
            l_lo = l_lo * f_lo + sum_lo;
            l_hi = l_hi * f_hi + sum_hi;
            if (__any_sync(0xffffffffu, f_lo != 1.f || f_hi != 1.f)) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    o[j][0] *= f_lo; o[j][1] *= f_lo;
                    o[j][2] *= f_hi; o[j][3] *= f_hi;
                }
            }
            // ---- O += P' V with P' = p * vs: two k-chunks of 16 tokens, 16 blocks of 8 channels, the first
            // eight of group 0 and the last eight of group 1
#pragma unroll
            for (int c16 = 0; c16 < 2; ++c16) {
                // scales of tokens 8 n8 + 2t and + 1 for n8 = 2 c16 (x) and 2 c16 + 1 (y)
                const uint2 va = *reinterpret_cast<const uint2*>(&sm_vs[par][16 * c16 + 2 * t]);
                const uint2 vc = *reinterpret_cast<const uint2*>(&sm_vs[par][16 * c16 + 8 + 2 * t]);
                uint32_t pa[2][4];
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const float a0 = __half2float(__ushort_as_half((unsigned short)(q ? va.x >> 16 : va.x & 0xffff)));
                    const float a1 = __half2float(__ushort_as_half((unsigned short)(q ? va.y >> 16 : va.y & 0xffff)));
                    const float c0 = __half2float(__ushort_as_half((unsigned short)(q ? vc.x >> 16 : vc.x & 0xffff)));
                    const float c1 = __half2float(__ushort_as_half((unsigned short)(q ? vc.y >> 16 : vc.y & 0xffff)));
                    pa[q][0] = pack_h2(s[2 * c16][0] * a0, s[2 * c16][1] * a1);
                    pa[q][1] = pack_h2(s[2 * c16][2] * a0, s[2 * c16][3] * a1);
                    pa[q][2] = pack_h2(s[2 * c16 + 1][0] * c0, s[2 * c16 + 1][1] * c1);
                    pa[q][3] = pack_h2(s[2 * c16 + 1][2] * c0, s[2 * c16 + 1][3] * c1);
                }
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {                  // two channel blocks per ldmatrix
                    constexpr int kHalf = 4;
                    const int q = jj / kHalf;
                    uint32_t bf[4];
                    ldsm_x4_trans(bf, vb + 16 * c16 * kVStride + 16 * jj);
                    mma_m16n8k16(o[2 * jj], pa[q][0], pa[q][1], pa[q][2], pa[q][3], bf[0], bf[1]);
                    mma_m16n8k16(o[2 * jj + 1], pa[q][0], pa[q][1], pa[q][2], pa[q][3], bf[2], bf[3]);
                }
            }
        }
        if (live[par ^ 1]) convert(par ^ 1, kw[par ^ 1], vw[par ^ 1], vsc[par ^ 1]);   // the next tile
        __syncthreads();
    };

    fetch(tile_begin, table_entry(tile_begin), kw[0], vw[0], vsc[0], live[0]);
    fetch(tile_begin + 1, table_entry(tile_begin + 1), kw[1], vw[1], vsc[1], live[1]);
    raw_ahead = table_entry(tile_begin + 2);
    // the first two tiles are on their way while the queries are prepared
    // ---- Q' = q * ks of all rows, high and low parts, stored order
    if (!idle) {
        const __half* ksp = p.ks + kvh * D;
        for (int idx = tid; idx < ROWS * NW; idx += kThreads) {
            const int row = idx / NW, c8 = idx % NW;
            __half hi[8], lo[8];
            if (row < rows_valid) {
                const __half* qp = p.q + int64_t(seq * p.m + row / rep) * p.q_stride + (kvh * rep + row % rep) * D + 8 * c8;
                __half qraw[8], sraw[8];
                *reinterpret_cast<uint4*>(sraw) = *reinterpret_cast<const uint4*>(ksp + 8 * c8);
                if ((reinterpret_cast<uintptr_t>(qp) & 15) == 0) {
                    *reinterpret_cast<uint4*>(qraw) = *reinterpret_cast<const uint4*>(qp);
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i) qraw[i] = qp[i];
                }
#pragma unroll
                for (int ps = 0; ps < 8; ++ps) {             // stored position ps holds natural channel ps/2 + 4 (ps%2)
                    const int i = (ps >> 1) + 4 * (ps & 1);
                    const float v = __half2float(qraw[i]) * __half2float(sraw[i]);      // exact in fp32
                    hi[ps] = __float2half_rn(v);
                    lo[ps] = __float2half_rn(v - __half2float(hi[ps]));
                }
            } else {
#pragma unroll
                for (int ps = 0; ps < 8; ++ps) hi[ps] = lo[ps] = __float2half_rn(0.f);
            }
            *reinterpret_cast<uint4*>(sm_qh + row * kVStride + 8 * c8) = *reinterpret_cast<const uint4*>(hi);
            *reinterpret_cast<uint4*>(sm_ql + row * kVStride + 8 * c8) = *reinterpret_cast<const uint4*>(lo);
        }
    }

    if (live[0]) convert(0, kw[0], vw[0], vsc[0]);
    __syncthreads();                                              // Q' and the first tile are in place
    for (int tile = tile_begin; tile < tile_end; tile += 2) {
        step(std::integral_constant<int, 0>{}, tile);
        if (tile + 1 < tile_end) step(std::integral_constant<int, 1>{}, tile + 1);
    }

    // ---- write-out.  o[j][0..1] is (row r_lo, stored columns 8j + 2t, 8j + 2t + 1) = natural channels
    // 8j + t and 8j + t + 4; o[j][2..3] the same for r_hi.
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
    if (mma_warp && !(idle && splits > 1)) {
#pragma unroll
        for (int hfr = 0; hfr < 2; ++hfr) {
            const int row = hfr ? r_hi : r_lo;
            if (row >= rows_valid) continue;
            const float den = hfr ? l_hi : l_lo, mx = hfr ? mx_hi : mx_lo;
            if (splits == 1) {
                const float inv = 1.f / fmaxf(den, 1e-20f);
                __half* dst = p.out + (int64_t(seq * p.m + row / rep) * p.hq + kvh * rep + row % rep) * D;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    dst[8 * j + t] = __float2half_rn(o[j][2 * hfr] * inv);
                    dst[8 * j + t + 4] = __float2half_rn(o[j][2 * hfr + 1] * inv);
                }
                if (t == 0 && p.lse)
                    p.lse[int64_t(seq * p.m + row / rep) * p.hq + kvh * rep + row % rep] = lse_of(mx, den);
            } else {
                float* dst = part + (int64_t(split) * rows_valid + row) * part_row(D);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    __stcg(dst + 8 * j + t, o[j][2 * hfr]);
                    __stcg(dst + 8 * j + t + 4, o[j][2 * hfr + 1]);
                }
                if (t == 0) { __stcg(dst + D, mx); __stcg(dst + D + 1, den); }
            }
        }
    }
    if (splits == 1) return;

    __threadfence();
    __syncthreads();
    int* counter = p.counters + seq * p.hkv + kvh;
    if (tid == 0) s_ticket = atomicAdd(counter, 1);
    __syncthreads();
    if (s_ticket != splits - 1) return;
    __threadfence();
    // the tile buffers are idle now: 64 rows x 64 splits pairs fit in them
    merge_splits<D, kThreads>(
        1, rows_valid, splits, reinterpret_cast<float2*>(sm_k), [&](int) { return part; },
        [&](int, int row, int d, const float4& acc, float inv, float lse) {
            store_h4(p.out + (int64_t(seq * p.m + row / rep) * p.hq + kvh * rep + row % rep) * D + d, acc, inv);
            if (d == 0 && p.lse) p.lse[int64_t(seq * p.m + row / rep) * p.hq + kvh * rep + row % rep] = lse;
        });
    if (tid == 0) *counter = 0;
}

// =====================================================================================
// Fast decode path: at most 8 query rows per KV head (one decode position of a GQA group
// of up to 8 heads, or a few verify positions), D in {64, 128}, at most two V groups.
//
// One CTA of 8 warps serves (sequence, split, group of `hpc` KV heads); warp w works on
// KV head w % hpc and on every (8/hpc)-th 32-token tile of the split.  Each warp keeps a
// private ring of cp.async stages (K rows, V rows) in shared memory, so the bytes in
// flight do not occupy registers and no CTA barrier is needed in the loop.
//
// Both products put the *cache* in the 16-row A operand of m16n8k16 and the (few) query
// rows in the 8-column B operand, so nothing is padded from 4 rows to 16:
//   S^T[token, row] = K[token, :] . Q'[row, :]     A = K nibbles, B = Q'^T
//   O^T[dim, row]  += V^T[dim, token] . P'[token, row]   A = V nibbles, B = P'^T
// Nibbles enter A as fp16 subnormals by masking alone (u * 2^-24, or 16u * 2^-24 for odd
// nibbles); the offsets and scales are applied outside the MMAs:
//   S  = 2^24 * acc - 8 * sum_d Q'[row, d]          (Q' = q * ks in two fp16 parts, /16 on odd slots)
//   O  = 2^24 * acc - 8 * sum_t P'[t, row],  P'[t, row] = p[t, row] * vs[t, group]
// P' is moved from the accumulator layout to the B layout with movmatrix.
// =====================================================================================
constexpr int kFastWarps = 8;
constexpr int kFastThreads = kFastWarps * 32;
constexpr int kFastTile = 32;                 // tokens per stage
constexpr int kFastStages = 3;

template <int D>
struct FastLayout {
    static constexpr int KROW = D / 2;                    // bytes per token row of one head
    static constexpr int VROW = D / 2 + 16;               // padded: conflict-free 32-bit column reads
    static constexpr int K_BYTES = kFastTile * KROW;
    static constexpr int V_BYTES = kFastTile * VROW;
    static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
    static constexpr int WARP_BYTES = kFastStages * STAGE_BYTES;
    static constexpr int RING_BYTES = kFastWarps * WARP_BYTES;
    static constexpr int MERGE_BYTES = kFastWarps * 8 * (D + 2) * 4;
    static constexpr int SMEM_BYTES = RING_BYTES > MERGE_BYTES ? RING_BYTES : MERGE_BYTES;
};

__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(d) : "r"(a));
    return d;
}


// PAIR (at most four query rows): the eight MMA columns hold, for row r, the high part of the fp16-split
// operand in column 2r and the low part in column 2r + 1, so lane t owns row t alone and both parts of a
// product come out of the same MMA.  Otherwise column n is row n, lane t owns rows 2t and 2t + 1, the low
// part of Q' takes a second MMA and P' stays one fp16.
template <int D, int NG, bool PAIR>
__global__ void __launch_bounds__(kFastThreads, 2) kv4_decode_fast_kernel(const AttnParams p, const int hpc) {
    pdl_launch_dependents();
    pdl_wait();
    using L = FastLayout<D>;
    constexpr int NW = D / 8;             // words per (token, head)
    constexpr int KWT = NW / 4;           // K words per lane per token
    constexpr int VW = NW / 8;            // V words per lane per token (word wsel*8 + g)
    constexpr int NO = 4 * VW;            // O accumulators per lane (each 16 dims x 8 columns)
    constexpr int KCH = D / 32;           // 16-byte chunks per lane per K (or V) tile
    constexpr int NR = PAIR ? 1 : 2;      // query rows per lane

    extern __shared__ __align__(16) unsigned char fsm[];
    __shared__ int s_ticket;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int wt = kFastWarps / hpc;                       // warps that share a head
    const int kvh = blockIdx.y * hpc + warp % hpc, ws = warp / hpc;
    const int split = blockIdx.x, seq = blockIdx.z;
    const int rep = p.hq / p.hkv;
    const int rows_valid = p.m * rep;

    const int capacity = p.max_blocks * p.page;
    const int len = p.lens[seq];
    const int reach = min(len + p.m - 1, capacity);
    const int tiles = reach > 0 ? (reach + kFastTile - 1) / kFastTile : 0;
    const int per_split = (tiles + p.splits - 1) / p.splits;
    const int tile_begin = split * per_split;
    const int tile_end = min(tiles, tile_begin + per_split);
    const int first = tile_begin + ws;
    const int n_my = first < tile_end ? (tile_end - first + wt - 1) / wt : 0;

    // Order of the prologue: the query and K-scale words are requested first (a few hundred bytes), then
    // the ring is started (block-table read, copies: the whole grid's first stages are ~19 MB, about 3 us of
    // HBM time), and the Q' fragments are computed from the words while those copies are in flight.  With
    // the ring started after the Q' set-up the two phases were serial; with the query loads behind the
    // copies they queue up behind 19 MB.
    const int qrow = PAIR ? (g >> 1) : g;
    const bool row_ok = qrow < rows_valid;
    uint4 q_words[KWT], s_words[KWT];
    {
        const int mrow = row_ok ? qrow / rep : 0;
        const __half* qp = p.q + int64_t(seq * p.m + mrow) * p.q_stride + (kvh * rep + (row_ok ? qrow % rep : 0)) * D;
        const __half* ksp = p.ks + kvh * D;
        const bool vec = (reinterpret_cast<uintptr_t>(qp) & 15) == 0;
#pragma unroll
        for (int wi = 0; wi < KWT; ++wi) {
            const int d0 = 8 * (t * KWT + wi);
            s_words[wi] = *reinterpret_cast<const uint4*>(ksp + d0);
            if (vec) {
                q_words[wi] = *reinterpret_cast<const uint4*>(qp + d0);
            } else {
                __half tmp[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) tmp[i] = qp[d0 + i];
                q_words[wi] = *reinterpret_cast<const uint4*>(tmp);
            }
        }
    }
    unsigned char* ring = fsm + warp * L::WARP_BYTES;
    const int64_t head_words = int64_t(p.hkv) * NW;
    uint32_t live_bits = 0;

    // lane-constant parts of the copy addresses: chunk c = lane + 32 j of a tile is
    // (token c / chunks_per_row, 16-byte part c % chunks_per_row)
    int64_t src_off[KCH];
    int kdst[KCH], vdst[KCH];
#pragma unroll
    for (int j = 0; j < KCH; ++j) {
        const int c = lane + 32 * j;
        const int tok = c / (L::KROW / 16), part = c % (L::KROW / 16);
        src_off[j] = tok * head_words + kvh * NW + part * 4;
        kdst[j] = tok * L::KROW + part * 16;
        vdst[j] = L::K_BYTES + tok * L::VROW + part * 16;
    }
    const __half* vs_lane = p.vs + (int64_t(lane) * p.hkv + kvh) * NG;
    const int32_t* bt_row = p.bt + int64_t(seq) * p.max_blocks;
    const int tiles_per_page = p.page / kFastTile;
    int cached_page = -1, cached_raw = -1;

    uint32_t sc_ring[kFastStages];
#pragma unroll
    for (int i = 0; i < kFastStages; ++i) sc_ring[i] = 0;

    auto issue = [&](int idx, int slot, uint32_t& sc) {
        const int tile = first + idx * wt;
        int page_idx, in_page;
        if (p.page_shift >= 0) {
            page_idx = (tile * kFastTile) >> p.page_shift;
            in_page = (tile * kFastTile) & (p.page - 1);
        } else {
            page_idx = tile / tiles_per_page;
            in_page = (tile - page_idx * tiles_per_page) * kFastTile;
        }
        if (page_idx != cached_page) {
            cached_page = page_idx;
            cached_raw = bt_row[page_idx];
        }
        const bool ok = cached_raw >= 0;
        live_bits = (live_bits & ~(1u << slot)) | (uint32_t(ok) << slot);
        if (!ok) return;
        const int64_t slot0 = int64_t(min(cached_raw, p.num_blocks - 1)) * p.page + in_page;
        unsigned char* dst = ring + slot * L::STAGE_BYTES;
        const uint32_t* ksrc = p.kq + slot0 * head_words;
        const uint32_t* vsrc = p.vq + slot0 * head_words;
#pragma unroll
        for (int j = 0; j < KCH; ++j) {
            cp_async_16(dst + kdst[j], ksrc + src_off[j]);
            cp_async_16(dst + vdst[j], vsrc + src_off[j]);
        }
        const __half* sp = vs_lane + slot0 * p.hkv * NG;
        sc = NG == 2 ? *reinterpret_cast<const uint32_t*>(sp) : uint32_t(__half_as_ushort(sp[0]));
    };

#pragma unroll
    for (int i = 0; i < kFastStages - 1; ++i) {
        if (i < n_my) issue(i, i, sc_ring[i]);
        cp_async_commit();
    }

    // ---- Q'^T fragments (B operand), column n = g; lane t covers words 4t..4t+3.
    // Q' = q * ks is exact in fp32 and is carried as a high and a low fp16 part: rounded to one fp16 it
    // would shift every score of the row by the same channel-wise error, which does not average out over
    // the tokens.
    uint32_t qb[KWT][2][2], ql[PAIR ? 1 : KWT][2][2];
    float qsum = 0.f;
    {
#pragma unroll
        for (int wi = 0; wi < KWT; ++wi) {
            __half qraw[8], sraw[8];
            *reinterpret_cast<uint4*>(sraw) = s_words[wi];
            *reinterpret_cast<uint4*>(qraw) = q_words[wi];
            __half qv[8], qw[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float v = row_ok ? __half2float(qraw[i]) * __half2float(sraw[i]) : 0.f;   // exact in fp32
                float hi = __half2float(__float2half_rn(v));
                float lo = __half2float(__float2half_rn(v - hi));
                if (PAIR) { hi = (g & 1) ? lo : hi; lo = 0.f; }
                // odd nibbles enter the A operand multiplied by 16
                qv[i] = __float2half_rn((i & 1) ? hi * 0.0625f : hi);
                qw[i] = __float2half_rn((i & 1) ? lo * 0.0625f : lo);
                qsum += ((i & 1) ? 16.f : 1.f) * (__half2float(qv[i]) + __half2float(qw[i]));
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                qb[wi][h][0] = h2_as_u32(__halves2half2(qv[2 * h], qv[2 * h + 4]));
                qb[wi][h][1] = h2_as_u32(__halves2half2(qv[2 * h + 1], qv[2 * h + 5]));
                if (!PAIR) {
                    ql[wi][h][0] = h2_as_u32(__halves2half2(qw[2 * h], qw[2 * h + 4]));
                    ql[wi][h][1] = h2_as_u32(__halves2half2(qw[2 * h + 1], qw[2 * h + 5]));
                }
            }
        }
    }
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 2);                 // sum over all D for column g
    const float c1 = 16777216.f * p.sl2;
    // rows of this lane: PAIR: row t (columns 2t, 2t+1 are its two parts); else rows 2t and 2t+1
    const int rw[2] = {PAIR ? t : 2 * t, PAIR ? t : 2 * t + 1};
    float cq[NR];
    int lim[NR];
    {
        const float qa = __shfl_sync(0xffffffffu, qsum, (2 * t) * 4), qc = __shfl_sync(0xffffffffu, qsum, (2 * t + 1) * 4);
        if (PAIR) {
            cq[0] = 8.f * p.sl2 * (qa + qc);
        } else {
            cq[0] = 8.f * p.sl2 * qa;
            cq[NR - 1] = 8.f * p.sl2 * qc;
        }
#pragma unroll
        for (int r = 0; r < NR; ++r) lim[r] = rw[r] < rows_valid ? min(len + rw[r] / rep, capacity) : 0;
    }
    // a padded (invalid) row is masked everywhere
    const int lim_min = rows_valid == (PAIR ? 4 : 8) ? min(len, capacity) : 0;

    float o[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[j][c] = 0.f;
    float mx[NR], l[NR], lp[NG][NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        mx[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int q = 0; q < NG; ++q) lp[q][r] = 0.f;
    }

    // The loop is unrolled over the ring so that the stage slot, its shared-memory address and
    // its entry of the register ring of scales are compile-time constants.
    for (int it0 = 0; it0 < n_my; it0 += kFastStages) {
#pragma unroll
      for (int slot = 0; slot < kFastStages; ++slot) {
        const int it = it0 + slot;
        if (it >= n_my) break;
        {
            const int nxt = it + kFastStages - 1;
            constexpr int kPrev = kFastStages - 1;
            const int nslot = (slot + kPrev) % kFastStages;
            uint32_t sc_new = 0;
            if (nxt < n_my) issue(nxt, nslot, sc_new);
            cp_async_commit();
            sc_ring[nslot] = sc_new;
        }
        cp_async_wait<kFastStages - 1>();
        __syncwarp();
        const uint32_t sc_cur = sc_ring[slot];
        if ((live_bits >> slot) & 1u) {
            const unsigned char* kb = ring + slot * L::STAGE_BYTES;
            const unsigned char* vb = kb + L::K_BYTES;
            const int pos0 = (first + it * wt) * kFastTile;
            // sv[b16][2 * tok + r]: token 16 b16 + g + 8 tok, row rw[r]
            float sv[2][2 * NR];
#pragma unroll
            for (int b16 = 0; b16 < 2; ++b16) {
                float acc[4] = {0.f, 0.f, 0.f, 0.f}, accl[4] = {0.f, 0.f, 0.f, 0.f};
                const int tokA = 16 * b16 + g, tokB = tokA + 8;
                uint32_t ka[KWT], kbw[KWT];
                if (KWT == 4) {
                    const uint4 x = *reinterpret_cast<const uint4*>(kb + tokA * L::KROW + t * 16);
                    const uint4 y = *reinterpret_cast<const uint4*>(kb + tokB * L::KROW + t * 16);
                    ka[0] = x.x; ka[1] = x.y; ka[KWT - 2] = x.z; ka[KWT - 1] = x.w;
                    kbw[0] = y.x; kbw[1] = y.y; kbw[KWT - 2] = y.z; kbw[KWT - 1] = y.w;
                } else {
                    const uint2 x = *reinterpret_cast<const uint2*>(kb + tokA * L::KROW + t * 8);
                    const uint2 y = *reinterpret_cast<const uint2*>(kb + tokB * L::KROW + t * 8);
                    ka[0] = x.x; ka[1] = x.y; kbw[0] = y.x; kbw[1] = y.y;
                }
#pragma unroll
                for (int wi = 0; wi < KWT; ++wi) {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t wa = ka[wi] >> (8 * h), wb = kbw[wi] >> (8 * h);
                        mma_m16n8k16(acc, wa & 0x000f000fu, wb & 0x000f000fu, wa & 0x00f000f0u, wb & 0x00f000f0u,
                                     qb[wi][h][0], qb[wi][h][1]);
                        if (!PAIR)
                            mma_m16n8k16(accl, wa & 0x000f000fu, wb & 0x000f000fu, wa & 0x00f000f0u, wb & 0x00f000f0u,
                                         ql[wi][h][0], ql[wi][h][1]);
                    }
                }
                if (PAIR) {
                    sv[b16][0] = fmaf(acc[0] + acc[1], c1, -cq[0]);
                    sv[b16][NR] = fmaf(acc[2] + acc[3], c1, -cq[0]);
                } else {
                    sv[b16][0] = fmaf(acc[0] + accl[0], c1, -cq[0]);
                    sv[b16][NR - 1] = fmaf(acc[1] + accl[1], c1, -cq[NR - 1]);
                    sv[b16][NR] = fmaf(acc[2] + accl[2], c1, -cq[0]);
                    sv[b16][2 * NR - 1] = fmaf(acc[3] + accl[3], c1, -cq[NR - 1]);
                }
                if (pos0 + kFastTile > lim_min) {            // warp-uniform: only the last tiles need masks
                    const int pa = pos0 + tokA, pb = pos0 + tokB;
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        if (pa >= lim[r]) sv[b16][r] = -INFINITY;
                        if (pb >= lim[r]) sv[b16][NR + r] = -INFINITY;
                    }
                }
            }
            float tm[NR], safe[NR], al[NR];
            bool moved = false;
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                tm[r] = fmaxf(fmaxf(sv[0][r], sv[0][NR + r]), fmaxf(sv[1][r], sv[1][NR + r]));
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) tm[r] = fmaxf(tm[r], __shfl_xor_sync(0xffffffffu, tm[r], off));
                const float n = fmaxf(mx[r], tm[r]);
                safe[r] = n == -INFINITY ? 0.f : n;
                al[r] = ex2(mx[r] - safe[r]);
                mx[r] = n;
                moved = moved || al[r] != 1.f;
            }
            if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    l[r] *= al[r];
#pragma unroll
                    for (int q = 0; q < NG; ++q) lp[q][r] *= al[r];
                }
                // accumulator columns 2t, 2t+1: both belong to row t (PAIR) or to rows 2t, 2t+1
#pragma unroll
                for (int j = 0; j < NO; ++j) {
                    o[j][0] *= al[0]; o[j][1] *= al[NR - 1]; o[j][2] *= al[0]; o[j][3] *= al[NR - 1];
                }
            }
            // The codes enter the MMAs as unsigned values, so the raw sums are large and positive while the
            // result (after the -8 * sum P' term) is small.  The tensor core truncates when it adds into its
            // accumulator; adding every tile into one long-lived accumulator would turn that into a bias that
            // grows with the context.  Each tile therefore starts fresh accumulators, which are added to the
            // running sums with ordinary (round-to-nearest) fp32 additions.
            float ot[NO][4];
#pragma unroll
            for (int b16 = 0; b16 < 2; ++b16) {
                float pr[2 * NR];
#pragma unroll
                for (int r = 0; r < NR; ++r) {
                    pr[r] = ex2(sv[b16][r] - safe[r]);
                    pr[NR + r] = ex2(sv[b16][NR + r] - safe[r]);
                    l[r] += pr[r] + pr[NR + r];
                }
                const uint32_t sA = __shfl_sync(0xffffffffu, sc_cur, 16 * b16 + g);
                const uint32_t sB = __shfl_sync(0xffffffffu, sc_cur, 16 * b16 + g + 8);
                const unsigned char* vrow = vb + (16 * b16) * L::VROW;
                const float2 fA = __half22float2(u32_as_h2(sA)), fB = __half22float2(u32_as_h2(sB));   // both groups' scales
#pragma unroll
                for (int q = 0; q < NG; ++q) {
                    const float fa = q ? fA.y : fA.x;
                    const float fb = q ? fB.y : fB.x;
                    // P' = p * vs enters the MMA as fp16: PAIR carries its rounding remainder in the odd column;
                    // otherwise it is one fp16.  The offset term -8 * sum P' must be summed from the same
                    // rounded values, or the rounding noise would enter the result multiplied by 8.
                    uint32_t h01, h23;
                    if (PAIR) {
                        // both tokens' parts in packed conversions
                        const float xa = pr[0] * fa, xb = pr[1] * fb;
                        const __half2 hab = __floats2half2_rn(xa, xb);
                        const float2 hf = __half22float2(hab);
                        const __half2 lab = __floats2half2_rn(xa - hf.x, xb - hf.y);
                        h01 = __byte_perm(h2_as_u32(hab), h2_as_u32(lab), 0x5410);       // (high, low) of token A
                        h23 = __byte_perm(h2_as_u32(hab), h2_as_u32(lab), 0x7632);       // of token B
                        const float2 lf = __half22float2(lab);
                        lp[q][0] += (hf.x + lf.x) + (hf.y + lf.y);
                    } else {
                        h01 = pack_h2(pr[0] * fa, pr[NR - 1] * fa);
                        h23 = pack_h2(pr[NR] * fb, pr[2 * NR - 1] * fb);
                        const float2 r01 = __half22float2(u32_as_h2(h01)), r23 = __half22float2(u32_as_h2(h23));
                        lp[q][0] += r01.x + r23.x;
                        lp[q][NR - 1] += r01.y + r23.y;
                    }
                    const uint32_t b0 = movmatrix_trans(h01);
                    const uint32_t b1 = movmatrix_trans(h23);
#pragma unroll
                    for (int wsel = (NG == 2 ? q : 0); wsel < (NG == 2 ? q + 1 : VW); ++wsel) {
                        const int wo = (wsel * 8 + g) * 4;
                        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(vrow + (2 * t) * L::VROW + wo);
                        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(vrow + (2 * t + 1) * L::VROW + wo);
                        const uint32_t w2 = *reinterpret_cast<const uint32_t*>(vrow + (2 * t + 8) * L::VROW + wo);
                        const uint32_t w3 = *reinterpret_cast<const uint32_t*>(vrow + (2 * t + 9) * L::VROW + wo);
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const uint32_t sel = b | (b << 4) | ((4 + b) << 8) | ((4 + b) << 12);
                            const uint32_t xa = __byte_perm(w0, w1, sel), xb = __byte_perm(w2, w3, sel);
                            if (b16 == 0)
                                mma_m16n8k16_zero(ot[wsel * 4 + b], xa & 0x000f000fu, xa & 0x00f000f0u, xb & 0x000f000fu,
                                                  xb & 0x00f000f0u, b0, b1);
                            else
                                mma_m16n8k16(ot[wsel * 4 + b], xa & 0x000f000fu, xa & 0x00f000f0u, xb & 0x000f000fu,
                                             xb & 0x00f000f0u, b0, b1);
                        }
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < NO; ++j)
#pragma unroll
                for (int c = 0; c < 4; ++c) o[j][c] += ot[j][c];
        }
        __syncwarp();
      }
    }
    cp_async_wait<0>();

    // ---- per-warp results; denominators and offset sums are summed over the 8 lane groups
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            l[r] += __shfl_xor_sync(0xffffffffu, l[r], off);
#pragma unroll
            for (int q = 0; q < NG; ++q) lp[q][r] += __shfl_xor_sync(0xffffffffu, lp[q][r], off);
        }
    }
    __syncthreads();                                   // all rings are idle: reuse them for the merge
    float* mo = reinterpret_cast<float*>(fsm) + warp * 8 * (D + 2);     // [8 rows][D + 2]
    // accumulator element c of o[j]: dimension `dim` (c < 2, codes times 2^-24) or `dim + 1` (c >= 2, the odd
    // nibble, codes times 2^-20); column 2t + (c & 1)
#pragma unroll
    for (int j = 0; j < NO; ++j) {
        const int wsel = j / 4, b = j % 4;
        const int grp = NG == 2 ? wsel : 0;
        const int dim = 8 * (wsel * 8 + g) + 2 * b;
        if (PAIR) {
            mo[rw[0] * (D + 2) + dim] = (o[j][0] + o[j][1]) * 16777216.f - 8.f * lp[grp][0];
            mo[rw[0] * (D + 2) + dim + 1] = (o[j][2] + o[j][3]) * 1048576.f - 8.f * lp[grp][0];
        } else {
            mo[rw[0] * (D + 2) + dim] = o[j][0] * 16777216.f - 8.f * lp[grp][0];
            mo[rw[1] * (D + 2) + dim] = o[j][1] * 16777216.f - 8.f * lp[grp][NR - 1];
            mo[rw[0] * (D + 2) + dim + 1] = o[j][2] * 1048576.f - 8.f * lp[grp][0];
            mo[rw[1] * (D + 2) + dim + 1] = o[j][3] * 1048576.f - 8.f * lp[grp][NR - 1];
        }
    }
    if (g == 0) {
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            mo[rw[r] * (D + 2) + D] = mx[r];
            mo[rw[r] * (D + 2) + D + 1] = l[r];
        }
    }
    __syncthreads();

    // ---- merge the wt warps of each head, then write the result or this split's partial
    const int splits = p.splits;
    const float* all = reinterpret_cast<const float*>(fsm);
    constexpr int D4 = D / 4;
    for (int e = tid; e < hpc * rows_valid * D4; e += kFastThreads) {
        const int d = (e % D4) * 4, hr = e / D4;
        const int hl = hr / rows_valid, row = hr - hl * rows_valid;
        const int head = blockIdx.y * hpc + hl;
        float mx = -INFINITY;
        for (int w = 0; w < wt; ++w) mx = fmaxf(mx, all[((w * hpc + hl) * 8 + row) * (D + 2) + D]);
        const float safe = mx == -INFINITY ? 0.f : mx;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        float den = 0.f;
        for (int w = 0; w < wt; ++w) {
            const float* src = all + ((w * hpc + hl) * 8 + row) * (D + 2);
            const float f = ex2(src[D] - safe);
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] += src[d + i] * f;
            den += src[D + 1] * f;
        }
        if (splits == 1) {
            const int mrow = row / rep, qh = head * rep + row % rep;
            const float inv = 1.f / fmaxf(den, 1e-20f);
            __half2 h01 = __floats2half2_rn(acc[0] * inv, acc[1] * inv), h23 = __floats2half2_rn(acc[2] * inv, acc[3] * inv);
            *reinterpret_cast<uint2*>(p.out + (int64_t(seq * p.m + mrow) * p.hq + qh) * D + d) =
                make_uint2(h2_as_u32(h01), h2_as_u32(h23));
        } else {
            float* dst = p.partial + ((int64_t(seq * p.hkv + head) * splits + split) * rows_valid + row) * part_row(D);
#pragma unroll
            for (int i = 0; i < 4; ++i) __stcg(dst + d + i, acc[i]);
            if (d == 0) { __stcg(dst + D, mx); __stcg(dst + D + 1, den); }
        }
    }
    if (splits == 1) return;

    __threadfence();
    __syncthreads();
    int* counter = p.counters + seq * gridDim.y + blockIdx.y;
    if (tid == 0) s_ticket = atomicAdd(counter, 1);
    __syncthreads();
    if (s_ticket != splits - 1) return;
    __threadfence();
    __syncthreads();                                   // the per-warp results in shared memory are consumed
    merge_splits<D, kFastThreads>(
        hpc, rows_valid, splits, reinterpret_cast<float2*>(fsm),
        [&](int hl) { return p.partial + (int64_t(seq * p.hkv + blockIdx.y * hpc + hl) * splits) * rows_valid * part_row(D); },
        [&](int hl, int row, int d, const float4& acc, float inv, float) {
            const int head = blockIdx.y * hpc + hl;
            store_h4(p.out + (int64_t(seq * p.m + row / rep) * p.hq + head * rep + row % rep) * D + d, acc, inv);
        });
    if (tid == 0) *counter = 0;
}

// KV heads per CTA for the fast path.  Measured at Qwen3-8B geometry: the best grids have
// about one resident wave of CTAs (two per SM) with as few splits as possible - batch 32 x
// 2.1 k tokens: 29 us with one head per CTA and no split against 32 us with two heads and two
// splits; batch 64 x 4 k: 85 us with two heads per CTA and no split against 100 us with eight
// heads and four splits.  So: the fewest heads per CTA whose grid still fits one wave.
int fast_heads_per_cta(int batch, int hkv, int64_t capacity) {
    (void)capacity;
    int hpc = 1;
    while (hpc < 8 && hkv % (hpc * 2) == 0 && int64_t(batch) * (hkv / hpc) > 2 * kNumSMs) hpc *= 2;
    return hpc;
}

bool fast_path_ok(int m, int hq, int hkv, int d, int page, int ng) {
    return m * (hq / hkv) <= 8 && page % kFastTile == 0 && (ng == 1 || (ng == 2 && d == 128));
}

constexpr int kMaxCounters = 1 << 16;

int row_tiles(int m, int hq, int hkv) {
    const int rt = cdiv(m * (hq / hkv), 16);
    return rt == 3 ? 4 : rt;
}

}  // namespace

int kv4_attention_splits(int batch, int m, int hq, int hkv, int d, int page, int max_blocks) {
    const int64_t capacity = int64_t(max_blocks) * page;
    // Shapes only.  Enough splits to fill one resident wave (two CTAs per SM), no warp longer
    // than 1024 tokens (so one long sequence in a batch cannot become the tail), never less
    // than 256 tokens of capacity per split.
    const bool fast = m * (hq / hkv) <= 8 && page % kFastTile == 0;
    int hpc, wt;
    if (fast) {
        hpc = fast_heads_per_cta(batch, hkv, capacity);
        wt = 8 / hpc;
    } else {                                             // 4-warp CTAs, one KV head each
        hpc = 1;
        wt = 2;
    }
    const int base = batch * (hkv / hpc);
    int64_t splits = (fast ? 2 : 4) * kNumSMs / base;    // floor: the grid stays within one resident wave
    int64_t by_len = cdiv64(capacity, int64_t(1024) * wt);
    // The verify kernel (one CTA walks its tokens alone, three CTAs per SM) is compute-bound.  Measured at
    // Qwen3-8B geometry with 2.2 k and 4.5 k tokens and batch 16 / 32 / 64, the time is flat within 5 % over
    // grids of two to three resident waves and rises outside: about 1024 CTAs, none shorter than 512 tokens.
    if (!fast && d == 128 && row_tiles(m, hq, hkv) >= 2 && page % kVTile == 0) {
        splits = cdiv64(1024, base);
        by_len = 1;
        const int64_t longest = capacity / 512 > 0 ? capacity / 512 : 1;
        if (splits > longest) splits = longest;
    }
    if (by_len > splits) splits = by_len;
    const int64_t most = capacity / 256 > 0 ? capacity / 256 : 1;
    if (splits > most) splits = most;
    if (splits > 64) splits = 64;
    if (splits < 1) splits = 1;
    return int(splits);
}

size_t kv4_attention_workspace_bytes(int batch, int m, int hq, int hkv, int d, int page, int max_blocks) {
    const int splits = kv4_attention_splits(batch, m, hq, hkv, d, page, max_blocks);
    size_t bytes = size_t(kMaxCounters) * sizeof(int);
    if (splits > 1) bytes += size_t(batch) * hq * m * splits * part_row(d) * sizeof(float);
    return bytes;
}

size_t kv4_attention_builtin_scratch_bytes() { return LQ2_BUILTIN_SCRATCH_BYTES; }

// Device address of the built-in scratch on the current device, resolved on the
// first call per device (this may load the module, so it must not happen while
// a stream is being captured) and remembered afterwards.
int kv4_attention_builtin_scratch(void** out) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return LQ2_ERR_CUDA;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_lq2_attention_scratch) != cudaSuccess || !p) return LQ2_ERR_CUDA;
        addr[dev] = p;
    }
    *out = addr[dev];
    return LQ2_OK;
}

size_t kv4_attention_counter_bytes(int batch, int hkv) { return size_t(batch) * hkv * sizeof(int); }

int kv4_attention_launch(const __half* q, int64_t q_stride, const uint32_t* kq, const __half* ks,
                         const uint32_t* vq, const __half* vs, const int32_t* bt, const int32_t* lens,
                         __half* out, float* lse, int pos_step, int batch, int m, int hq, int hkv, int d, int page, int max_blocks,
                         int v_group, int64_t num_slots, void* workspace, size_t workspace_bytes,
                         cudaStream_t st) {
    if (batch * hkv > kMaxCounters) return LQ2_ERR_SHAPE;
    if (!workspace || workspace_bytes < kv4_attention_workspace_bytes(batch, m, hq, hkv, d, page, max_blocks))
        return LQ2_ERR_WORKSPACE;
    AttnParams p;
    p.q = q; p.q_stride = q_stride; p.kq = kq; p.ks = ks; p.vq = vq; p.vs = vs; p.bt = bt; p.lens = lens;
    p.lse = lse; p.pos_step = pos_step;
    p.out = out; p.batch = batch; p.m = m; p.hq = hq; p.hkv = hkv; p.page = page; p.max_blocks = max_blocks;
    p.ng = d / v_group;
    int shift = 0;
    while ((1 << shift) < v_group) ++shift;
    p.vg_shift = shift;
    p.num_blocks = int(num_slots / page);
    p.page_shift = -1;
    for (int sft = 0; sft < 31; ++sft)
        if ((1 << sft) == page) p.page_shift = sft;
    p.splits = kv4_attention_splits(batch, m, hq, hkv, d, page, max_blocks);
    p.sl2 = float(1.4426950408889634 / sqrt(double(d)));
    p.counters = reinterpret_cast<int*>(workspace);
    p.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + size_t(kMaxCounters) * sizeof(int));
    if (fast_path_ok(m, hq, hkv, d, page, p.ng) && pos_step == 1 && !lse) {
        const int hpc = fast_heads_per_cta(batch, hkv, int64_t(max_blocks) * page);
        dim3 fgrid(p.splits, hkv / hpc, batch);
        static bool configured[64] = {};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LQ2_ERR_CUDA;
        const bool pair = m * (hq / hkv) <= 4;
#define LQ2_FAST_ATTR(DD, GG, PP) \
    (cudaFuncSetAttribute(kv4_decode_fast_kernel<DD, GG, PP>, cudaFuncAttributeMaxDynamicSharedMemorySize, FastLayout<DD>::SMEM_BYTES) == cudaSuccess)
#define LQ2_FAST(DD, GG, PP) \
    return launch_pdl(kv4_decode_fast_kernel<DD, GG, PP>, fgrid, dim3(kFastThreads), FastLayout<DD>::SMEM_BYTES, st, 1, p, hpc)
        if (!configured[dev]) {
            const bool ok = LQ2_FAST_ATTR(128, 1, true) && LQ2_FAST_ATTR(128, 2, true) && LQ2_FAST_ATTR(64, 1, true) &&
                            LQ2_FAST_ATTR(128, 1, false) && LQ2_FAST_ATTR(128, 2, false) && LQ2_FAST_ATTR(64, 1, false);
            if (!ok) return LQ2_ERR_CUDA;
            configured[dev] = true;
        }
        if (pair) {
            if (d == 128 && p.ng == 2) LQ2_FAST(128, 2, true);
            if (d == 128) LQ2_FAST(128, 1, true);
            LQ2_FAST(64, 1, true);
        }
        if (d == 128 && p.ng == 2) LQ2_FAST(128, 2, false);
        if (d == 128) LQ2_FAST(128, 1, false);
        LQ2_FAST(64, 1, false);
#undef LQ2_FAST
#undef LQ2_FAST_ATTR
    }
    const int rt = row_tiles(m, hq, hkv);
    dim3 grid(p.splits, hkv, batch);
    if (d == 128 && rt >= 2 && page % kVTile == 0 && p.ng <= 2) {
        static bool verify_ready[64] = {};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LQ2_ERR_CUDA;
        if (!verify_ready[dev]) {
            if (cudaFuncSetAttribute(kv4_verify_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, VerifyLayout<2>::SMEM_BYTES) != cudaSuccess ||
                cudaFuncSetAttribute(kv4_verify_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, VerifyLayout<4>::SMEM_BYTES) != cudaSuccess)
                return LQ2_ERR_CUDA;
            verify_ready[dev] = true;
        }
        if (rt == 2) return launch_pdl(kv4_verify_kernel<2>, grid, dim3(kThreads), VerifyLayout<2>::SMEM_BYTES, st, 1, p);
        return launch_pdl(kv4_verify_kernel<4>, grid, dim3(kThreads), VerifyLayout<4>::SMEM_BYTES, st, 1, p);
    }
#define LQ2_ATTN(DD, RR) return launch_pdl(kv4_attention_kernel<DD, RR>, grid, dim3(kThreads), 0, st, 1, p)
    if (d == 128) {
        if (rt == 1) LQ2_ATTN(128, 1); else if (rt == 2) LQ2_ATTN(128, 2); else LQ2_ATTN(128, 4);
    } else {
        if (rt == 1) LQ2_ATTN(64, 1); else if (rt == 2) LQ2_ATTN(64, 2); else LQ2_ATTN(64, 4);
    }
#undef LQ2_ATTN
}


}  // namespace lq2
