// Paged attention over the int4 KV pool: decode (one query position) and
// multi-position verify, split-KV flash-decoding with an online softmax.
//
// Replaces paged_attention_decode and its three Triton kernels
// (qslab/kernels/kv4/paged_attention.py:11-150: decode kernel, split merge and
// launcher; qslab/kernels/kv4/grouped_attention.py:7-63: grouped verify).
//
// Work decomposition.  One CTA serves one (sequence, KV head, split): all query
// heads of the GQA group — and for verify all M positions — share a single read
// of the packed K/V bytes.  Query rows are ordered row = m * rep + head_in_group
// and cut into tiles of 16; warp w works on row tile w % RT and, when RT < 4, on
// every (4/RT)-th 16-token block of the split.  Both products run on the
// warp-level tensor-core op m16n8k16 with fp32 accumulation:
//   S = Q' K^T : Q' = fp16(q * ks) carries the static per-channel K scale, so K
//                enters as the exact integers (nibble - 8);
//   O += P V   : V is dequantised to fp16 (nibble - 8) * vs rounded once, as the
//                reference's verify kernel does (grouped_attention.py:50-53).
// Nibbles are unpacked in registers in an order that needs one shift per word;
// the matching permutation of head channels is applied to Q' once at load and to
// O once at the write-out.  Scores, the running maximum, the denominator and O
// stay fp32.
//
// Splits.  The split count depends on shapes only.  Each CTA writes an fp32
// partial (O, max, denominator) per row, takes a ticket, and the last CTA of a
// (sequence, KV head) merges the partials in split order and writes fp16.
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
    int splits;
    float sl2;  // D^-0.5 * log2(e)
    float* partial;
    int* counters;
};

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

// RT: 16-row query tiles per (sequence, KV head): ceil(M * rep / 16), 3 rounded up to 4.
template <int D, int RT>
__global__ void __launch_bounds__(kThreads) kv4_attention_kernel(const AttnParams p) {
    constexpr int NW = D / 8;          // words per (token, head)
    constexpr int KWT = NW / 4;        // K words per lane per token (lanes t = 0..3 split the row)
    constexpr int VWT = NW / 8;        // V words per lane per token (lanes g = 0..7 split the row)
    constexpr int NT = 8 * VWT;        // n-tiles (of 8 channels) of the PV product per lane
    constexpr int WT = kWarps / RT;    // warps that split the tokens of one row tile
    constexpr int ROWS = 16 * RT;
    using KW = typename KWords<D>::type;
    using VW = typename VWords<D>::type;

    __shared__ float sm_o[kWarps][16][D];
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
    const int reach = min(len + p.m - 1, capacity);          // keys any row of this sequence reads
    const int tiles = reach > 0 ? (reach + kTile - 1) / kTile : 0;
    const int per_split = (tiles + p.splits - 1) / p.splits;
    const int tile_begin = split * per_split;
    const int tile_end = min(tiles, tile_begin + per_split);

    // ---- Q' fragments: rows r_lo = 16*rt + g and r_hi = r_lo + 8
    const int r_lo = 16 * rt + g, r_hi = r_lo + 8;
    const bool v_lo = r_lo < rows_valid, v_hi = r_hi < rows_valid;
    const int m_lo = v_lo ? r_lo / rep : 0, m_hi = v_hi ? r_hi / rep : 0;
    const int lim_lo = v_lo ? min(len + m_lo, capacity) : 0;
    const int lim_hi = v_hi ? min(len + m_hi, capacity) : 0;
    uint32_t qa[KWT][2][4];
    {
        const __half* q_lo = p.q + int64_t(seq * p.m + m_lo) * p.q_stride + (kvh * rep + (v_lo ? r_lo % rep : 0)) * D;
        const __half* q_hi = p.q + int64_t(seq * p.m + m_hi) * p.q_stride + (kvh * rep + (v_hi ? r_hi % rep : 0)) * D;
        const __half* ksp = p.ks + kvh * D;
#pragma unroll
        for (int wi = 0; wi < KWT; ++wi) {
            const int d0 = 8 * (t * KWT + wi);
            float sc[8], lo[8], hi[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                sc[i] = __half2float(ksp[d0 + i]);
                lo[i] = v_lo ? __half2float(q_lo[d0 + i]) * sc[i] : 0.f;
                hi[i] = v_hi ? __half2float(q_hi[d0 + i]) * sc[i] : 0.f;
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                qa[wi][h][0] = pack_h2(lo[2 * h], lo[2 * h + 4]);
                qa[wi][h][1] = pack_h2(hi[2 * h], hi[2 * h + 4]);
                qa[wi][h][2] = pack_h2(lo[2 * h + 1], lo[2 * h + 5]);
                qa[wi][h][3] = pack_h2(hi[2 * h + 1], hi[2 * h + 5]);
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
            float s[2][4];
#pragma unroll
            for (int n8 = 0; n8 < 2; ++n8) {
#pragma unroll
                for (int c = 0; c < 4; ++c) s[n8][c] = 0.f;
#pragma unroll
                for (int wi = 0; wi < KWT; ++wi) {
                    const uint32_t w = word_of(kw[n8], wi);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t x = w >> (8 * h);
                        const uint32_t b0 = h2_as_u32(__hsub2(u32_as_h2(and_or(x, 0x000f000fu, 0x64006400u)), k1032));
                        const uint32_t b1 = h2_as_u32(__hfma2(u32_as_h2(and_or(x, 0x00f000f0u, 0x64006400u)), k16th, km72));
                        mma_m16n8k16(s[n8], qa[wi][h][0], qa[wi][h][1], qa[wi][h][2], qa[wi][h][3], b0, b1);
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
                    const float v = pos < lim ? s[n8][c] * p.sl2 : -INFINITY;
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
    float* part = p.partial + (int64_t(seq * p.hkv + kvh) * splits) * rows_valid * (D + 2);
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
        } else {
            float* dst = part + (int64_t(split) * rows_valid + row) * (D + 2);
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
    for (int e = tid; e < rows_valid * D; e += kThreads) {
        const int row = e / D, d = e % D;
        float mx = -INFINITY;
        for (int sp = 0; sp < splits; ++sp)
            mx = fmaxf(mx, __ldcg(part + (int64_t(sp) * rows_valid + row) * (D + 2) + D));
        const float safe = mx == -INFINITY ? 0.f : mx;
        float acc = 0.f, den = 0.f;
        for (int sp = 0; sp < splits; ++sp) {
            const float* src = part + (int64_t(sp) * rows_valid + row) * (D + 2);
            const float f = exp2f(__ldcg(src + D) - safe);
            acc += __ldcg(src + d) * f;
            den += __ldcg(src + D + 1) * f;
        }
        const int mrow = row / rep, head = kvh * rep + row % rep;
        p.out[(int64_t(seq * p.m + mrow) * p.hq + head) * D + d] = __float2half_rn(acc / fmaxf(den, 1e-20f));
    }
    if (tid == 0) *counter = 0;
}

constexpr int kMaxCounters = 1 << 16;

int row_tiles(int m, int hq, int hkv) {
    const int rt = cdiv(m * (hq / hkv), 16);
    return rt == 3 ? 4 : rt;
}

}  // namespace

int kv4_attention_splits(int batch, int m, int hq, int hkv, int d, int page, int max_blocks) {
    (void)d; (void)m; (void)hq;
    const int64_t capacity = int64_t(max_blocks) * page;
    const int base = batch * hkv;
    // Enough CTAs to fill the machine three times over, and no CTA longer than
    // 4096 tokens so that one long sequence in a batch cannot become the tail;
    // never less than 256 tokens of capacity per split.
    int64_t splits = cdiv(3 * kNumSMs, base);
    const int64_t by_len = cdiv64(capacity, 4096);
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
    if (splits > 1) bytes += size_t(batch) * hq * m * splits * (d + 2) * sizeof(float);
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
                         __half* out, int batch, int m, int hq, int hkv, int d, int page, int max_blocks,
                         int v_group, int64_t num_slots, void* workspace, size_t workspace_bytes,
                         cudaStream_t st) {
    if (batch * hkv > kMaxCounters) return LQ2_ERR_SHAPE;
    if (!workspace || workspace_bytes < kv4_attention_workspace_bytes(batch, m, hq, hkv, d, page, max_blocks))
        return LQ2_ERR_WORKSPACE;
    AttnParams p;
    p.q = q; p.q_stride = q_stride; p.kq = kq; p.ks = ks; p.vq = vq; p.vs = vs; p.bt = bt; p.lens = lens;
    p.out = out; p.batch = batch; p.m = m; p.hq = hq; p.hkv = hkv; p.page = page; p.max_blocks = max_blocks;
    p.ng = d / v_group;
    int shift = 0;
    while ((1 << shift) < v_group) ++shift;
    p.vg_shift = shift;
    p.num_blocks = int(num_slots / page);
    p.splits = kv4_attention_splits(batch, m, hq, hkv, d, page, max_blocks);
    p.sl2 = float(1.4426950408889634 / sqrt(double(d)));
    p.counters = reinterpret_cast<int*>(workspace);
    p.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + size_t(kMaxCounters) * sizeof(int));
    const int rt = row_tiles(m, hq, hkv);
    dim3 grid(p.splits, hkv, batch);
#define LQ2_ATTN(DD, RR) kv4_attention_kernel<DD, RR><<<grid, kThreads, 0, st>>>(p)
    if (d == 128) {
        if (rt == 1) LQ2_ATTN(128, 1); else if (rt == 2) LQ2_ATTN(128, 2); else LQ2_ATTN(128, 4);
    } else {
        if (rt == 1) LQ2_ATTN(64, 1); else if (rt == 2) LQ2_ATTN(64, 2); else LQ2_ATTN(64, 4);
    }
#undef LQ2_ATTN
    return check_launch();
}

}  // namespace lq2
