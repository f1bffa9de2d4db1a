/*
 * linkq2_b200 — C ABI of the B200 (sm_100a) W4A16 and KV4 operators.
 *
 * Every entry point takes raw device pointers, sizes, element strides and a
 * CUDA stream (a cudaStream_t passed as void*), enqueues its kernels on that
 * stream and returns at once.  The return value is LQ2_OK or an LQ2_ERR_* code
 * describing which argument was rejected; a rejected call launches nothing.
 *
 * The compute entry points allocate nothing, free nothing, never synchronise
 * and keep no state between calls.  The exceptions, each marked below:
 *   - two process-wide switches, lq2_w4a16_set_constant_weights and
 *     lq2_allreduce_set_poll_limit (a launch uses the value at launch time);
 *   - the tensor-parallel setup calls lq2_allreduce_buffer_create/open/close,
 *     which allocate, map and free device memory and synchronise;
 *   - lq2_allreduce_timeouts, which synchronises to read a device counter;
 *   - lq2_kv4_attention_static, whose scratch is one array inside the library
 *     that keeps the previous call's contents.
 *
 * Paths cited below are relative to the LinkQ2 project root and name the
 * reference interface each function stands in for.
 */
#ifndef LINKQ2_B200_H
#define LINKQ2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LQ2_OK 0
#define LQ2_ERR_ARG 1        /* null pointer or non-positive size */
#define LQ2_ERR_SHAPE 2      /* shape the operator does not support */
#define LQ2_ERR_ALIGN 3      /* pointer or stride misaligned for vector access */
#define LQ2_ERR_WORKSPACE 4  /* workspace missing or smaller than *_workspace_bytes */
#define LQ2_ERR_CUDA 5       /* the launch itself was refused by the CUDA runtime */
#define LQ2_ERR_LIMIT 6      /* lq2_kv4_attention_static: scratch need exceeds the built-in buffer */

/* Human-readable text for a status code. */
const char* lq2_status_string(int status);

/* ABI revision; bumped whenever a signature below changes. */
int lq2_abi_version(void);

/* --------------------------------------------------------------------------
 * W4A16 linear
 * -------------------------------------------------------------------------- */

/*
 * Load-time packing, replacing pack_weights_over_cols_triton(codes, 4, 32,
 * transpose=True).contiguous() and the "+8" of symmetric checkpoints
 * (qslab/kernels/gemlite/bitpack.py:96-125, qslab/runtime/backends/gemlite.py:22-25).
 *
 *   values  [N, K] int8   logical checkpoint integers (-8..7 symmetric, 0..15 affine)
 *   offset  8 for symmetric checkpoints, 0 for affine ones
 *   packed  [K/8, N] int32, n fastest: word(k8, n) = sum_j (values[n, 8*k8+j] + offset) << 4j
 * K must be a multiple of 8.
 */
int lq2_w4_pack(const int8_t* values, int offset, int32_t* packed, int n, int k, void* stream);

/*
 * Declares the quantized weights constant (enabled != 0) or not (0, the
 * default); returns the previous setting.  Process-wide.  No counterpart in
 * the reference.
 *
 * Every kernel of this library is launched with programmatic stream
 * serialization: it may be scheduled while the previous kernel of the stream is
 * draining and waits for that kernel's completion before touching activations or
 * outputs, so stream order is preserved for them.  With constant weights declared,
 * lq2_w4a16_linear additionally starts fetching packed/scales/zeros BEFORE that
 * wait.  The caller then guarantees that no kernel launched immediately before a
 * lq2_w4a16_linear call on the same stream writes its packed, scales or zeros
 * buffers - true for any inference loop once the checkpoint is loaded (the
 * runtime enables it after loading; a memcpy, an event wait, a synchronize or
 * any other kernel in between also restores the ordering).
 */
int lq2_w4a16_set_constant_weights(int enabled);

/*
 * Bytes of scratch lq2_w4a16_linear needs for this problem size.  The current
 * kernels keep split-K partials on chip and need none (the answer is 0 and the
 * workspace argument may be NULL); the query stays in the ABI so that a caller
 * written against it keeps working if a later kernel needs scratch again.  A
 * non-empty buffer must be zero-filled once when it is created.
 */
size_t lq2_w4a16_workspace_bytes(int m, int n, int k);

/*
 * y[M, N] = x[M, K] . dequant(W)^T, replacing qslab.kernels.gemlite.ops.linear
 * and its three Triton routes (qslab/kernels/gemlite/ops.py:10-15;
 * triton_kernels/gemv_revsplitK_A16fWnO16f_int32packing.py:155-384,
 * gemm_splitK_A16fWnO16f_int32packing.py:199-412, gemm_A16fWnO16f_int32packing.py:174-373)
 * with W_group_mode 3 dequantisation (u - z) * s (triton_kernels/utils.py:66-71).
 *
 *   x          [M, K] fp16, row stride x_row_stride elements, unit inner stride
 *   packed     [K/8, N] int32 (layout of lq2_w4_pack)
 *   scales     [K/group, N] fp16
 *   zeros      [K/group, N] fp16 per-group zero points, or NULL for the
 *              symmetric scalar zero 8
 *   y          [M, N] fp16 contiguous
 *   group      power of two >= 32 dividing K;  N a multiple of 32
 *   workspace  lq2_w4a16_workspace_bytes(M, N, K) bytes (see above); NULL when that is 0
 * Products are accumulated in fp32 and rounded to fp16 once.
 */
int lq2_w4a16_linear(const void* x, int64_t x_row_stride, const int32_t* packed,
                     const void* scales, const void* zeros, void* y, int m, int n, int k,
                     int group, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The gate and up projections of Qwen3MLP and the activation between them in one launch,
 * replacing F.silu(gate_proj(x)) * up_proj(x) (qslab/runtime/model/qwen3.py:59-64):
 *   y[M, N/2][m, 4b + j] = fp16(silu(fp32(g))) * u,  g = z[m, 8b + j], u = z[m, 8b + 4 + j],
 *   z = fp16(x . dequant(W)^T) as lq2_w4a16_linear would have written it.
 * packed / scales / zeros are the two projections' buffers with their columns interleaved in
 * blocks of four, [g0..g3 | u0..u3 | g4..g7 | u4..u7 | ...] (a load-time layout step on the
 * [K/8, N] buffers, nothing is repacked); N = 2 * intermediate size, a multiple of 64.
 * Other arguments as lq2_w4a16_linear.
 */
int lq2_w4a16_gate_up_silu(const void* x, int64_t x_row_stride, const int32_t* packed,
                           const void* scales, const void* zeros, void* y, int m, int n, int k,
                           int group, void* workspace, size_t workspace_bytes, void* stream);

/* --------------------------------------------------------------------------
 * KV4 cache.  Pool layout (qslab/runtime/execute/model_runner.py:146-156):
 *   kq, vq  [S, HKV, D/8] 32-bit words, 8 offset-binary nibbles per word
 *   ks      [HKV, D] fp16 static per-channel K scale
 *   vs      [S, HKV, D/v_group] fp16 per-token per-group V scale
 * -------------------------------------------------------------------------- */

/*
 * Quantize and scatter one batch of tokens, replacing store_kv_quant
 * (qslab/kernels/kv4/store.py:9-68).  slot -1 skips the token; any other slot
 * outside [0, num_slots) is skipped as well instead of being written.
 *
 *   k, v       [T, HKV, D] fp16; token stride k_stride / v_stride elements,
 *              head stride D, unit inner stride (slices of a fused QKV buffer work)
 *   slots      [T] int32
 * D a multiple of 8, v_group a multiple of 8 dividing D.
 */
int lq2_kv4_store(const void* k, const void* v, int64_t k_stride, int64_t v_stride,
                  uint32_t* kq, const void* ks, uint32_t* vq, void* vs, const int32_t* slots,
                  int tokens, int hkv, int d, int v_group, int64_t num_slots, void* stream);

/*
 * The same for fp32 keys and values: the reference's kernel converts whatever element
 * type it is given to fp32 before it quantizes (store.py:31,45), and its own tests store
 * fp32 tensors (tests/kernels/test_kv4_verify.py:98-102), so fp32 inputs are quantized
 * from their full precision, not rounded to fp16 first.  Strides in fp32 elements.
 */
int lq2_kv4_store_f32(const float* k, const float* v, int64_t k_stride, int64_t v_stride,
                      uint32_t* kq, const void* ks, uint32_t* vq, void* vs, const int32_t* slots,
                      int tokens, int hkv, int d, int v_group, int64_t num_slots, void* stream);

/*
 * Number of KV splits lq2_kv4_attention will use.  It depends on shapes only
 * (never on device values), so a captured CUDA graph stays valid
 * (same property as qslab/kernels/kv4/paged_attention.py:127-131).
 */
int lq2_kv4_attention_splits(int batch, int verify_m, int hq, int hkv, int d, int page,
                             int max_blocks);

/* Scratch bytes for lq2_kv4_attention; same zero-fill contract as the W4A16 workspace. */
size_t lq2_kv4_attention_workspace_bytes(int batch, int verify_m, int hq, int hkv, int d,
                                         int page, int max_blocks);

/*
 * Paged attention over the int4 pool for one query position per sequence
 * (verify_m == 1) or verify_m consecutive positions, replacing
 * paged_attention_decode and its kernels
 * (qslab/kernels/kv4/paged_attention.py:11-150,
 * qslab/kernels/kv4/grouped_attention.py:7-63).
 *
 *   q             [batch*verify_m, HQ, D] fp16, row stride q_row_stride elements
 *   block_tables  [batch, max_blocks] int32, negative entries are padding
 *   context_lens  [batch] int32; row seq*verify_m + m attends to logical
 *                 positions [0, context_lens[seq] + m) capped at max_blocks*page
 *   out           [batch*verify_m, HQ, D] fp16 contiguous
 * Positions under a negative block-table entry are masked; a row without any
 * valid position yields zeros.  Block ids are clamped into the pool's whole pages
 * ([0, floor(num_slots/page)); the pool need not be a multiple of the page, as the
 * reference's own tests allocate it) before any address is formed.
 * D must be 64 or 128, HQ a multiple of HKV with verify_m*HQ/HKV <= 64,
 * page a multiple of 16.
 */
int lq2_kv4_attention(const void* q, int64_t q_row_stride, const uint32_t* kq, const void* ks,
                      const uint32_t* vq, const void* vs, const int32_t* block_tables,
                      const int32_t* context_lens, void* out, int batch, int verify_m, int hq,
                      int hkv, int d, int page, int max_blocks, int v_group, int64_t num_slots,
                      void* workspace, size_t workspace_bytes, void* stream);

/*
 * Attention of blocks of new rows over the pool-resident prefix only: every row of block b attends to
 * positions [0, prefix_lens[b]) of the block table row b, with no causal step between the rows, and the
 * natural-log sum of exp(scaled scores) of each row is returned beside the normalised output so that the
 * caller can merge it with the attention over the rows' own (fp16) keys.  This is the pool half of the
 * chunked-prefill attention that the reference builds from materialize_kv + torch.cat + flash-attn
 * (qslab/runtime/model/attention.py:38-56,119-131): the prefix is read as int4 and never written back
 * as fp16.
 *
 *   q             [blocks*rows, HQ, D] fp16, row stride q_row_stride elements
 *   block_tables  [blocks, max_blocks] int32 (the sequence's row, repeated for each of its blocks)
 *   prefix_lens   [blocks] int32
 *   out           [blocks*rows, HQ, D] fp16;  lse [blocks*rows, HQ] fp32 (-inf for a row without keys)
 * rows*HQ/HKV must be in 9..64; workspace as for lq2_kv4_attention with (blocks, rows) in place of
 * (batch, verify_m).
 */
int lq2_kv4_attention_prefix(const void* q, int64_t q_row_stride, const uint32_t* kq, const void* ks,
                             const uint32_t* vq, const void* vs, const int32_t* block_tables,
                             const int32_t* prefix_lens, void* out, float* lse, int blocks, int rows,
                             int hq, int hkv, int d, int page, int max_blocks, int v_group,
                             int64_t num_slots, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Causal attention of a prefill step's new rows over the fp16 K/V of the same step, merged with the
 * prefix part that lq2_kv4_attention_prefix returned; with it, the step's attention no longer needs the
 * restored fp16 prefix nor the flash-attn call of qslab/runtime/model/attention.py:119-131.
 *
 *   q [rows, HQ, D], k, v [rows, HKV, D] fp16, row strides in elements (views into a fused projection
 *       output are fine: k rows 16-byte aligned, v rows 8-byte aligned)
 *   first_row   [rows] int32: first row of the step that belongs to the same sequence; row i attends to
 *               rows first_row[i] .. i
 *   prefix_row  [rows] int32: row of (pre, pre_lse) that holds this row's prefix part, -1 when its sequence
 *               has no prefix, -2 to leave the row of `out` untouched
 *   pre [*, HQ, D] fp16, pre_lse [*, HQ] fp32 (natural log); may be NULL when no row refers to them
 *   out [rows, HQ, D] fp16 contiguous
 * D is 64 or 128, HQ / HKV at most 8.
 */
int lq2_chunk_attention(const void* q, int64_t q_row_stride, const void* k, int64_t k_row_stride, const void* v,
                        int64_t v_row_stride, const int32_t* first_row, const int32_t* prefix_row,
                        const void* pre, const float* pre_lse, void* out, int rows, int hq, int hkv, int d,
                        void* stream);

/*
 * lq2_kv4_attention for callers that cannot allocate device memory.  It has no
 * counterpart in the reference.
 *
 * Some hosts of this library never get to call cudaMalloc: a plugin loaded into
 * a serving process that owns the whole device through its own pool and passes
 * the plugin nothing but the request's tensors, or code that runs where an
 * allocation would stall the device or is forbidden outright.  For them the
 * split partials and ticket counters live in a 16 MiB array compiled into the
 * library (lq2_kv4_attention_static_max_bytes() returns the size); every GPU
 * that loads the library keeps that array until the process exits.  Arguments
 * and results are those of lq2_kv4_attention without the workspace pair; the
 * same kernel runs, so the output is identical.
 *
 *  - A problem whose lq2_kv4_attention_workspace_bytes() exceeds the array is
 *    refused with LQ2_ERR_LIMIT and launches nothing.
 *  - The first call on each device looks up the array's device address; make
 *    that first call outside any stream capture.
 *  - All calls on a device share the one array.  Each call clears the counters
 *    it uses on its stream before the kernel, so calls issued one after another
 *    are independent, but two calls that may run at the same time on one GPU
 *    (different streams) race on it.
 *  - The call itself performs no cudaMalloc, cudaFree or other allocation.
 */
int lq2_kv4_attention_static(const void* q, int64_t q_row_stride, const uint32_t* kq, const void* ks,
                             const uint32_t* vq, const void* vs, const int32_t* block_tables,
                             const int32_t* context_lens, void* out, int batch, int verify_m, int hq,
                             int hkv, int d, int page, int max_blocks, int v_group,
                             int64_t num_slots, void* stream);

/* Size in bytes of the array behind lq2_kv4_attention_static. */
size_t lq2_kv4_attention_static_max_bytes(void);

/*
 * Prefix restore: gather the given slots and dequantise them to fp16
 * [T, HKV, D], replacing materialize_kv (qslab/kernels/kv4/layout.py:9-47).
 * Order of slots is kept and duplicates are allowed.  Each value is
 * fp16(fp32(nibble - 8) * fp32(scale)).  Slots outside [0, num_slots) produce zeros.
 */
int lq2_kv4_materialize(const uint32_t* kq, const void* ks, const uint32_t* vq, const void* vs,
                        const int64_t* slots, void* k_out, void* v_out, int tokens, int hkv,
                        int d, int v_group, int64_t num_slots, void* stream);

/* --------------------------------------------------------------------------
 * Fused elementwise steps between the operators above.  The reference runs
 * them as eager torch kernels; these keep its rounding points (fp32 statistics
 * and rotation, fp16 casts and fp16 products where torch has them).
 * -------------------------------------------------------------------------- */

/*
 * RMSNorm with optional residual add, replacing RMSNorm.forward
 * (qslab/runtime/model/primitives.py:15-36).
 *   residual == NULL:  out = fp16(x32 * rsqrt(mean(x32^2) + eps)) * weight
 *   residual != NULL:  s = fp32(x) + fp32(residual); residual_out = fp16(s);
 *                      out = fp16(s * rsqrt(mean(s^2) + eps)) * weight
 * x [rows, hidden] fp16 with row stride x_row_stride; residual, out,
 * residual_out contiguous [rows, hidden]; residual_out may alias residual.
 * hidden a multiple of 8, at most 8192.
 */
int lq2_rmsnorm(const void* x, int64_t x_row_stride, const void* residual, const void* weight,
                void* out, void* residual_out, int rows, int hidden, float eps, void* stream);

/*
 * out = fp16(silu(fp32(gate))) * up, replacing F.silu(gate) * up of Qwen3MLP.forward
 * (qslab/runtime/model/qwen3.py:64).  gate/up [rows, width] fp16 with row
 * strides; out contiguous.
 */
int lq2_silu_mul(const void* gate, int64_t gate_row_stride, const void* up, int64_t up_row_stride,
                 void* out, int rows, int width, void* stream);

/*
 * Everything between the q/k/v projections and the attention kernel in one
 * launch: per-head RMSNorm of q and k, rotary embedding, SmoothAttention scaling
 * and the KV4 store, replacing qslab/runtime/model/qwen3.py:49-51,
 * rotary.py:12-16,103-108, attention.py:72-77 and :102-110 (store_kv_quant).
 *   q [T, HQ, D], k, v [T, HKV, D] fp16, token strides in elements, head stride D
 *   q_norm_weight, k_norm_weight [D] fp16;  cos_sin [max_pos, D] fp32, cos in
 *   the first D/2 columns and sin in the last (the reference's cos_sin_cache);
 *   positions [T] int64;  lam_q [HQ, D], lam_k [HKV, D] fp16 or NULL (lambda = 1)
 *   q_out [T, HQ, D] fp16 contiguous;  k_out [T, HKV, D] fp16 or NULL: the
 *   rotated, scaled keys for callers that also need them in fp16 (prefill)
 *   kq, ks, vq, vs, slots, v_group, num_slots as in lq2_kv4_store; slots == NULL
 *   skips the store.
 * The cache bytes equal lq2_kv4_store applied to (k_out, v).  D is 64 or 128.
 */
int lq2_pre_attention(const void* q, const void* k, const void* v, int64_t q_stride, int64_t k_stride,
                      int64_t v_stride, const void* q_norm_weight, const void* k_norm_weight,
                      const float* cos_sin, const int64_t* positions, const void* lam_q,
                      const void* lam_k, void* q_out, void* k_out, uint32_t* kq, const void* ks,
                      uint32_t* vq, void* vs, const int32_t* slots, int tokens, int hq, int hkv, int d,
                      int v_group, int64_t num_slots, float eps, void* stream);

/*
 * Fills the fixed input buffers of a captured decode graph for one step, replacing the
 * seven device copies of CUDAGraphs.replay (qslab/runtime/execute/cuda_graph.py:60-72).
 * packed (device, int32): [batch ids | batch positions | batch slots | batch context
 * lengths | batch x width block-table entries].  Rows batch..rows_cap-1 get slot -1 and
 * context length 0, table entries outside [batch, width] get 0, as the reference pads.
 * input_ids, positions [rows_cap] int64; slot_mapping, context_lens [rows_cap] int32;
 * block_tables [rows_cap, width_cap] int32.
 */
int lq2_stage_decode(const int32_t* packed, int64_t* input_ids, int64_t* positions, int32_t* slot_mapping,
                     int32_t* context_lens, int32_t* block_tables, int batch, int rows_cap, int width,
                     int width_cap, void* stream);

/* --------------------------------------------------------------------------
 * Tensor-parallel exchange.  No counterpart in the reference, which is
 * single-GPU (qslab/runtime/model/qwen3.py:1-5): the sum all-reduce of the
 * [M, hidden] fp16 activations that the row-split o_proj and down_proj
 * (qwen3.py:53,64) need when the layers are sharded over the GPUs of one
 * NVSwitch domain, one process per GPU.  One kernel per rank over peer memory;
 * a message is pushed into every peer's buffer and summed there in rank order
 * (fp32), so all ranks obtain identical bits.
 *
 * Setup, once per process: every rank creates one exchange buffer, hands its
 * 64-byte handle to the other ranks (any host channel), opens theirs, and
 * passes the table of world pointers, its own at index rank, to every call.
 * All ranks must issue the same sequence of lq2_allreduce_fp16 calls (same
 * counts), each rank on one stream.  These setup calls are the only entry
 * points of the library that allocate device memory or synchronise.
 * -------------------------------------------------------------------------- */

/* Size of the exchange buffer for `world` ranks (2..8) and messages of up to
 * max_message_bytes (a multiple of 16); 0 for unsupported arguments. */
size_t lq2_allreduce_buffer_bytes(int world, size_t max_message_bytes);

/* Allocates (cudaMalloc) and zero-fills this rank's buffer on the current device
 * and writes its CUDA IPC handle (64 bytes) to ipc_handle_64. */
int lq2_allreduce_buffer_create(size_t bytes, void** buffer, void* ipc_handle_64);

/* Maps a peer's buffer from its handle (peer access is enabled on demand). */
int lq2_allreduce_buffer_open(const void* ipc_handle_64, void** buffer);

/* Unmaps a peer's buffer (own == 0) or frees this rank's (own != 0). */
int lq2_allreduce_buffer_close(void* buffer, int own);

/*
 * out[i] = sum over ranks of x[i], i < count (fp16; count * 2 a multiple of 16 and at most
 * max_message_bytes, else LQ2_ERR_SHAPE / LQ2_ERR_LIMIT).  out may alias x.
 * buffers: host array of `world` device pointers (this rank's own buffer at index rank).
 * Waits inside the kernel are bounded; a peer that never arrives is counted in
 * lq2_allreduce_timeouts() instead of hanging the GPU (the output is then invalid).
 */
int lq2_allreduce_fp16(const void* x, void* out, int64_t count, void* const* buffers, int rank, int world,
                       size_t max_message_bytes, void* stream);

/*
 * The all-reduce above followed by the residual RMSNorm of lq2_rmsnorm, in one launch:
 *   h = fp16(sum over ranks of x);  s = fp32(h) + fp32(residual);  residual_out = fp16(s);
 *   out = fp16(s * rsqrt(mean(s^2) + eps)) * weight
 * i.e. tp.all_reduce(o_proj(...)) / tp.all_reduce(down_proj(...)) and the layer norm that
 * consumes it (qslab/runtime/model/qwen3.py:53,64 with primitives.py:23-30).  x [rows, hidden]
 * is this rank's partial sum (row stride x_row_stride); rows * hidden * 2 must not exceed
 * max_message_bytes (LQ2_ERR_LIMIT).  Counts as one call in the sequence all ranks share.
 */
int lq2_rmsnorm_allreduce(const void* x, int64_t x_row_stride, const void* residual, const void* weight, void* out,
                          void* residual_out, int rows, int hidden, float eps, void* const* buffers, int rank,
                          int world, size_t max_message_bytes, void* stream);

/*
 * The producer side of the same exchange fused into the projection: lq2_w4a16_linear for a
 * row-split o_proj / down_proj (8 < M <= 64, else LQ2_ERR_SHAPE) whose epilogue, besides writing
 * this rank's partial sum to y, stores every finished group of four outputs directly into the
 * peers' exchange buffers in the flagged form lq2_rmsnorm_allreduce gathers, so the transfer
 * over NVLink runs while the rest of the projection is still being computed.  It must be
 * followed, as the next exchange call on every rank, by lq2_rmsnorm_allreduce_pushed on y:
 * the same as lq2_rmsnorm_allreduce except that it only gathers (nothing is sent again).
 * M * N * 2 must not exceed max_message_bytes (LQ2_ERR_LIMIT).
 */
int lq2_w4a16_linear_push(const void* x, int64_t x_row_stride, const int32_t* packed, const void* scales,
                          const void* zeros, void* y, int m, int n, int k, int group, void* const* buffers, int rank,
                          int world, size_t max_message_bytes, void* stream);
int lq2_rmsnorm_allreduce_pushed(const void* x, int64_t x_row_stride, const void* residual, const void* weight,
                                 void* out, void* residual_out, int rows, int hidden, float eps, void* const* buffers,
                                 int rank, int world, size_t max_message_bytes, void* stream);

/* Number of abandoned waits on the current device since the library was loaded
 * (synchronises the device); 0 in a healthy run. */
unsigned int lq2_allreduce_timeouts(void);

/*
 * How long a thread of the exchange kernels waits for its peers: `polls` looks at the
 * exchange buffer in total per thread and launch, over all the pieces it waits for
 * (<= 0 restores the default, 2^22, a few seconds).  Process-wide; a launch (or a
 * captured graph node) keeps the value it was issued with.  Returns the previous value.
 * A thread that runs out stops waiting, the kernel completes with an invalid result and
 * lq2_allreduce_timeouts() counts it: a peer that has left costs seconds, not a hang.
 */
long long lq2_allreduce_set_poll_limit(long long polls);

#ifdef __cplusplus
}
#endif
#endif /* LINKQ2_B200_H */
