// extern "C" surface of the library: argument validation, then a launch.
// Declarations and the contract of each entry point are in include/linkq2_b200.h.
#include "common.cuh"

namespace lq2 {
int w4_pack_launch(const int8_t*, int, int32_t*, int, int, cudaStream_t);
size_t w4a16_stream_workspace_bytes(int, int, int);
int w4a16_stream_launch(const __half*, int64_t, const int32_t*, const __half*, const __half*, __half*,
                        int, int, int, int, int, void*, size_t, cudaStream_t);
int w4a16_umma_launch(const __half*, int64_t, const int32_t*, const __half*, const __half*, __half*, int, int,
                      int, int, int, const PushTarget*, cudaStream_t);
int kv4_store_launch(const __half*, const __half*, int64_t, int64_t, uint32_t*, const __half*, uint32_t*,
                     __half*, const int32_t*, int, int, int, int, int64_t, cudaStream_t);
int kv4_store_f32_launch(const float*, const float*, int64_t, int64_t, uint32_t*, const __half*, uint32_t*,
                         __half*, const int32_t*, int, int, int, int, int64_t, cudaStream_t);
int kv4_materialize_launch(const uint32_t*, const __half*, const uint32_t*, const __half*, const int64_t*,
                           __half*, __half*, int, int, int, int, int64_t, cudaStream_t);
int kv4_attention_splits(int, int, int, int, int, int, int);
size_t kv4_attention_workspace_bytes(int, int, int, int, int, int, int);
int kv4_attention_launch(const __half*, int64_t, const uint32_t*, const __half*, const uint32_t*,
                         const __half*, const int32_t*, const int32_t*, __half*, float*, int, int, int, int, int, int,
                         int, int, int, int64_t, void*, size_t, cudaStream_t);
int chunk_attention_launch(const __half*, int64_t, const __half*, int64_t, const __half*, int64_t, const int32_t*,
                           const int32_t*, const __half*, const float*, __half*, int, int, int, int, cudaStream_t);
size_t kv4_attention_builtin_scratch_bytes();
int kv4_attention_builtin_scratch(void**);
size_t kv4_attention_counter_bytes(int, int);
}  // namespace lq2

using namespace lq2;

#include <atomic>
#include <cstdlib>

namespace {
std::atomic<int> g_constant_weights{0};
}  // namespace

namespace lq2 {
bool early_weight_fetch() { return g_constant_weights.load(std::memory_order_relaxed) != 0; }
bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("LQ2_DISABLE_PDL");
        return !(v && v[0] == '1');
    }();
    return on;
}
}  // namespace lq2

namespace {
inline bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
inline bool w4_shape_ok(int m, int n, int k, int group) {
    return m > 0 && n > 0 && k > 0 && n % 32 == 0 && group >= 32 && pow2(group) && k % group == 0;
}
inline bool attn_shape_ok(int batch, int m, int hq, int hkv, int d, int page, int max_blocks) {
    return batch > 0 && m > 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && (d == 64 || d == 128) &&
           page > 0 && page % 16 == 0 && max_blocks > 0 && m * (hq / hkv) <= 64;
}
}  // namespace

extern "C" {

const char* lq2_status_string(int status) {
    switch (status) {
        case LQ2_OK: return "ok";
        case LQ2_ERR_ARG: return "null pointer or non-positive size";
        case LQ2_ERR_SHAPE: return "unsupported shape";
        case LQ2_ERR_ALIGN: return "pointer or stride not aligned for vector access";
        case LQ2_ERR_WORKSPACE: return "workspace missing or too small";
        case LQ2_ERR_CUDA: return "CUDA launch failed";
        case LQ2_ERR_LIMIT: return "problem needs more scratch than the built-in 16 MiB buffer";
        default: return "unknown status";
    }
}

int lq2_abi_version(void) { return 1; }

int lq2_w4_pack(const int8_t* values, int offset, int32_t* packed, int n, int k, void* stream) {
    if (!values || !packed || n <= 0 || k <= 0) return LQ2_ERR_ARG;
    if (k % 8 || (offset != 0 && offset != 8)) return LQ2_ERR_SHAPE;
    if (!aligned(values, 8) || !aligned(packed, 4)) return LQ2_ERR_ALIGN;
    return w4_pack_launch(values, offset, packed, n, k, static_cast<cudaStream_t>(stream));
}

int lq2_w4a16_set_constant_weights(int enabled) {
    return g_constant_weights.exchange(enabled ? 1 : 0, std::memory_order_relaxed);
}

size_t lq2_w4a16_workspace_bytes(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    return w4a16_stream_workspace_bytes(m, n, k);
}

namespace {
int w4a16_dispatch(const void* x, int64_t x_row_stride, const int32_t* packed, const void* scales,
                   const void* zeros, void* y, int m, int n, int k, int group, int silu, void* workspace,
                   size_t workspace_bytes, void* stream, const PushTarget* push = nullptr) {
    if (!x || !packed || !scales || !y) return LQ2_ERR_ARG;
    if (!w4_shape_ok(m, n, k, group)) return m <= 0 || n <= 0 || k <= 0 ? LQ2_ERR_ARG : LQ2_ERR_SHAPE;
    if (!aligned(x, 16) || x_row_stride % 8 || x_row_stride < k || !aligned(packed, 16) ||
        !aligned(scales, 16) || (zeros && !aligned(zeros, 16)) || !aligned(y, 8))
        return LQ2_ERR_ALIGN;
    // up to 8 rows: the weight-streaming kernel; beyond that the tcgen05 kernel
    if (push && (m <= 8 || m > 64)) return LQ2_ERR_SHAPE;
    if (m > 8)
        return w4a16_umma_launch(static_cast<const __half*>(x), x_row_stride, packed,
                                 static_cast<const __half*>(scales), static_cast<const __half*>(zeros),
                                 static_cast<__half*>(y), m, n, k, group, silu, push,
                                 static_cast<cudaStream_t>(stream));
    return w4a16_stream_launch(static_cast<const __half*>(x), x_row_stride, packed,
                               static_cast<const __half*>(scales), static_cast<const __half*>(zeros),
                               static_cast<__half*>(y), m, n, k, group, silu, workspace, workspace_bytes,
                               static_cast<cudaStream_t>(stream));
}
}  // namespace

int lq2_w4a16_linear(const void* x, int64_t x_row_stride, const int32_t* packed, const void* scales,
                     const void* zeros, void* y, int m, int n, int k, int group, void* workspace,
                     size_t workspace_bytes, void* stream) {
    return w4a16_dispatch(x, x_row_stride, packed, scales, zeros, y, m, n, k, group, 0, workspace, workspace_bytes,
                          stream);
}

int lq2_w4a16_linear_push(const void* x, int64_t x_row_stride, const int32_t* packed, const void* scales,
                          const void* zeros, void* y, int m, int n, int k, int group, void* const* buffers, int rank,
                          int world, size_t max_message_bytes, void* stream) {
    if (!buffers) return LQ2_ERR_ARG;
    if (world < 2 || world > kMaxWorld || rank < 0 || rank >= world || max_message_bytes % 16) return LQ2_ERR_SHAPE;
    if (m > 0 && n > 0 && size_t(m) * n * 2 > max_message_bytes) return LQ2_ERR_LIMIT;
    PushTarget push;
    for (int p = 0; p < kMaxWorld; ++p) {
        push.peers.base[p] = p < world ? static_cast<unsigned char*>(buffers[p]) : nullptr;
        if (p < world && !push.peers.base[p]) return LQ2_ERR_ARG;
    }
    push.rank = rank;
    push.world = world;
    push.max_bytes = max_message_bytes;
    return w4a16_dispatch(x, x_row_stride, packed, scales, zeros, y, m, n, k, group, 0, nullptr, 0, stream, &push);
}

int lq2_w4a16_gate_up_silu(const void* x, int64_t x_row_stride, const int32_t* packed, const void* scales,
                           const void* zeros, void* y, int m, int n, int k, int group, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (n % 64) return n > 0 ? LQ2_ERR_SHAPE : LQ2_ERR_ARG;
    return w4a16_dispatch(x, x_row_stride, packed, scales, zeros, y, m, n, k, group, 1, workspace, workspace_bytes,
                          stream);
}

int lq2_kv4_store(const void* k, const void* v, int64_t k_stride, int64_t v_stride, uint32_t* kq,
                  const void* ks, uint32_t* vq, void* vs, const int32_t* slots, int tokens, int hkv,
                  int d, int v_group, int64_t num_slots, void* stream) {
    if (tokens == 0) return LQ2_OK;
    if (!k || !v || !kq || !ks || !vq || !vs || !slots || tokens < 0 || hkv <= 0 || d <= 0 || num_slots <= 0)
        return LQ2_ERR_ARG;
    if (d % 8 || v_group < 8 || v_group > 256 || !pow2(v_group) || d % v_group) return LQ2_ERR_SHAPE;
    if (!aligned(ks, 16) || !aligned(k, 2) || !aligned(v, 2)) return LQ2_ERR_ALIGN;
    return kv4_store_launch(static_cast<const __half*>(k), static_cast<const __half*>(v), k_stride,
                            v_stride, kq, static_cast<const __half*>(ks), vq, static_cast<__half*>(vs),
                            slots, tokens, hkv, d, v_group, num_slots, static_cast<cudaStream_t>(stream));
}

int lq2_kv4_store_f32(const float* k, const float* v, int64_t k_stride, int64_t v_stride, uint32_t* kq,
                      const void* ks, uint32_t* vq, void* vs, const int32_t* slots, int tokens, int hkv,
                      int d, int v_group, int64_t num_slots, void* stream) {
    if (tokens == 0) return LQ2_OK;
    if (!k || !v || !kq || !ks || !vq || !vs || !slots || tokens < 0 || hkv <= 0 || d <= 0 || num_slots <= 0)
        return LQ2_ERR_ARG;
    if (d % 8 || v_group < 8 || v_group > 256 || !pow2(v_group) || d % v_group) return LQ2_ERR_SHAPE;
    if (!aligned(ks, 16) || !aligned(k, 4) || !aligned(v, 4)) return LQ2_ERR_ALIGN;
    return kv4_store_f32_launch(k, v, k_stride, v_stride, kq, static_cast<const __half*>(ks), vq,
                                static_cast<__half*>(vs), slots, tokens, hkv, d, v_group, num_slots,
                                static_cast<cudaStream_t>(stream));
}

int lq2_kv4_attention_splits(int batch, int verify_m, int hq, int hkv, int d, int page, int max_blocks) {
    if (!attn_shape_ok(batch, verify_m, hq, hkv, d, page, max_blocks)) return 0;
    return kv4_attention_splits(batch, verify_m, hq, hkv, d, page, max_blocks);
}

size_t lq2_kv4_attention_workspace_bytes(int batch, int verify_m, int hq, int hkv, int d, int page,
                                         int max_blocks) {
    if (!attn_shape_ok(batch, verify_m, hq, hkv, d, page, max_blocks)) return 0;
    return kv4_attention_workspace_bytes(batch, verify_m, hq, hkv, d, page, max_blocks);
}

int lq2_kv4_attention(const void* q, int64_t q_row_stride, const uint32_t* kq, const void* ks,
                      const uint32_t* vq, const void* vs, const int32_t* block_tables,
                      const int32_t* context_lens, void* out, int batch, int verify_m, int hq, int hkv,
                      int d, int page, int max_blocks, int v_group, int64_t num_slots, void* workspace,
                      size_t workspace_bytes, void* stream) {
    if (batch == 0) return LQ2_OK;
    if (!q || !kq || !ks || !vq || !vs || !block_tables || !context_lens || !out || num_slots <= 0)
        return LQ2_ERR_ARG;
    if (!attn_shape_ok(batch, verify_m, hq, hkv, d, page, max_blocks)) return LQ2_ERR_SHAPE;
    if (v_group < d / 8 || !pow2(v_group) || d % v_group || num_slots < page) return LQ2_ERR_SHAPE;
    if (!aligned(kq, 16) || !aligned(vq, 16) || !aligned(q, 2) || !aligned(workspace, 16)) return LQ2_ERR_ALIGN;
    return kv4_attention_launch(static_cast<const __half*>(q), q_row_stride, kq,
                                static_cast<const __half*>(ks), vq, static_cast<const __half*>(vs),
                                block_tables, context_lens, static_cast<__half*>(out), nullptr, 1, batch, verify_m, hq,
                                hkv, d, page, max_blocks, v_group, num_slots, workspace, workspace_bytes,
                                static_cast<cudaStream_t>(stream));
}

int lq2_kv4_attention_prefix(const void* q, int64_t q_row_stride, const uint32_t* kq, const void* ks,
                             const uint32_t* vq, const void* vs, const int32_t* block_tables,
                             const int32_t* prefix_lens, void* out, float* lse, int blocks, int rows, int hq,
                             int hkv, int d, int page, int max_blocks, int v_group, int64_t num_slots,
                             void* workspace, size_t workspace_bytes, void* stream) {
    if (blocks == 0) return LQ2_OK;
    if (!q || !kq || !ks || !vq || !vs || !block_tables || !prefix_lens || !out || !lse || num_slots <= 0)
        return LQ2_ERR_ARG;
    if (!attn_shape_ok(blocks, rows, hq, hkv, d, page, max_blocks)) return LQ2_ERR_SHAPE;
    if (rows * (hq / hkv) <= 8) return LQ2_ERR_SHAPE;          // blocks of at least 9 query rows per KV head
    if (v_group < d / 8 || !pow2(v_group) || d % v_group || num_slots < page) return LQ2_ERR_SHAPE;
    if (!aligned(kq, 16) || !aligned(vq, 16) || !aligned(q, 2) || !aligned(workspace, 16) || !aligned(lse, 4))
        return LQ2_ERR_ALIGN;
    return kv4_attention_launch(static_cast<const __half*>(q), q_row_stride, kq,
                                static_cast<const __half*>(ks), vq, static_cast<const __half*>(vs),
                                block_tables, prefix_lens, static_cast<__half*>(out), lse, 0, blocks, rows, hq,
                                hkv, d, page, max_blocks, v_group, num_slots, workspace, workspace_bytes,
                                static_cast<cudaStream_t>(stream));
}

int lq2_chunk_attention(const void* q, int64_t q_row_stride, const void* k, int64_t k_row_stride, const void* v,
                        int64_t v_row_stride, const int32_t* first_row, const int32_t* prefix_row, const void* pre,
                        const float* pre_lse, void* out, int rows, int hq, int hkv, int d, void* stream) {
    if (rows == 0) return LQ2_OK;
    if (!q || !k || !v || !first_row || !prefix_row || !out || rows < 0) return LQ2_ERR_ARG;
    if ((d != 64 && d != 128) || hkv <= 0 || hq <= 0 || hq % hkv || hq / hkv > 8) return LQ2_ERR_SHAPE;
    if (k_row_stride % 8 || v_row_stride % 4 || !aligned(k, 16) || !aligned(v, 8) || !aligned(q, 2) ||
        !aligned(out, 4) || !aligned(pre, 4) || !aligned(pre_lse, 4))
        return LQ2_ERR_ALIGN;
    return chunk_attention_launch(static_cast<const __half*>(q), q_row_stride, static_cast<const __half*>(k),
                                  k_row_stride, static_cast<const __half*>(v), v_row_stride, first_row, prefix_row,
                                  static_cast<const __half*>(pre), pre_lse, static_cast<__half*>(out), rows, hq, hkv,
                                  d, static_cast<cudaStream_t>(stream));
}

size_t lq2_kv4_attention_static_max_bytes(void) { return kv4_attention_builtin_scratch_bytes(); }

int lq2_kv4_attention_static(const void* q, int64_t q_row_stride, const uint32_t* kq, const void* ks,
                             const uint32_t* vq, const void* vs, const int32_t* block_tables,
                             const int32_t* context_lens, void* out, int batch, int verify_m, int hq,
                             int hkv, int d, int page, int max_blocks, int v_group, int64_t num_slots,
                             void* stream) {
    if (batch == 0) return LQ2_OK;
    if (!attn_shape_ok(batch, verify_m, hq, hkv, d, page, max_blocks)) return LQ2_ERR_SHAPE;
    if (v_group < d / 8 || !pow2(v_group) || d % v_group || num_slots < page) return LQ2_ERR_SHAPE;
    const size_t need = kv4_attention_workspace_bytes(batch, verify_m, hq, hkv, d, page, max_blocks);
    if (need > kv4_attention_builtin_scratch_bytes()) return LQ2_ERR_LIMIT;
    if (!q || !kq || !ks || !vq || !vs || !block_tables || !context_lens || !out) return LQ2_ERR_ARG;
    if (!aligned(kq, 16) || !aligned(vq, 16) || !aligned(q, 2)) return LQ2_ERR_ALIGN;
    void* scratch = nullptr;
    const int st = kv4_attention_builtin_scratch(&scratch);
    if (st != LQ2_OK) return st;
    // The array keeps whatever the previous call left; the ticket counters must
    // start at zero, so clear the ones this call will use (a stream-ordered
    // memset, not an allocation).
    if (cudaMemsetAsync(scratch, 0, kv4_attention_counter_bytes(batch, hkv),
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return LQ2_ERR_CUDA;
    return lq2_kv4_attention(q, q_row_stride, kq, ks, vq, vs, block_tables, context_lens, out, batch,
                             verify_m, hq, hkv, d, page, max_blocks, v_group, num_slots, scratch,
                             kv4_attention_builtin_scratch_bytes(), stream);
}

int lq2_kv4_materialize(const uint32_t* kq, const void* ks, const uint32_t* vq, const void* vs,
                        const int64_t* slots, void* k_out, void* v_out, int tokens, int hkv, int d,
                        int v_group, int64_t num_slots, void* stream) {
    if (tokens == 0) return LQ2_OK;
    if (!kq || !ks || !vq || !vs || !slots || !k_out || !v_out || tokens < 0 || hkv <= 0 || d <= 0 || num_slots <= 0)
        return LQ2_ERR_ARG;
    if (d % 8 || v_group < 8 || !pow2(v_group) || d % v_group) return LQ2_ERR_SHAPE;
    if (!aligned(ks, 16) || !aligned(k_out, 16) || !aligned(v_out, 16)) return LQ2_ERR_ALIGN;
    return kv4_materialize_launch(kq, static_cast<const __half*>(ks), vq, static_cast<const __half*>(vs),
                                  slots, static_cast<__half*>(k_out), static_cast<__half*>(v_out), tokens,
                                  hkv, d, v_group, num_slots, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
