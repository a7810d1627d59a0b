/*
 * h3b.h — C ABI of libh3b.so, the B200 (sm_100a) kernels behind the LOSSLESS
 * packed-Ulysses DiT block of H3-Flash.
 *
 * Every entry point:
 *   - takes raw device pointers, element counts and element strides (no
 *     framework types), plus the CUDA stream to enqueue on;
 *   - is stream-ordered: it never synchronises the host and never allocates;
 *   - returns H3B_OK (0) or an error code; h3b_last_error() then returns a
 *     message for the calling thread.
 * Tensors are bf16 (IEEE bfloat16 bit patterns) unless stated; RoPE tables are
 * fp32; AdaLN table indices are int64. Strides are in elements.
 *
 * Each declaration names the reference interface it replaces
 * (fluxmatrix/h3-flash, paths relative to the project root).
 */
#ifndef H3B_H_
#define H3B_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* h3b_stream_t; /* == cudaStream_t */

#define H3B_OK 0
#define H3B_ERR_VALUE 1       /* bad shape / argument: Python raises ValueError   */
#define H3B_ERR_CUDA 2        /* CUDA launch or driver error: RuntimeError         */
#define H3B_ERR_UNSUPPORTED 3 /* valid input this build does not handle: RuntimeError */

#define H3B_ABI_VERSION 8

int h3b_abi_version(void);
/* Kernels launched through this library by this process (all devices and host
 * threads), counted at launch; h3b_reset_kernel_launches sets it back to 0.
 * No reference counterpart: instrumentation for benchmarks and tests. */
int64_t h3b_kernel_launches(void);
void h3b_reset_kernel_launches(void);
/* Message of the last failing call on this host thread ("" if none). */
const char* h3b_last_error(void);

/* Device-side status word shared by all kernels of this library on the current
 * device. Bounded waits inside kernels that time out OR a bit into it instead of
 * spinning forever. h3b_device_status() copies it to the host (synchronous);
 * h3b_clear_device_status() zeroes it (stream-ordered). Bits:
 *   1 = attention pipeline wait timed out;
 *   2 = h3b_peer_barrier gave up waiting for a peer (10 s);
 *   4 = QKV GEMM pipeline wait timed out. */
int h3b_device_status(int* status_out);
int h3b_clear_device_status(h3b_stream_t stream);

/* ---------------------------------------------------------------------------
 * AdaLN / norm elementwise ops. Rows are `rows` vectors of `cols` values.
 * `index` holds `n_index` int64 table-row ids; row r reads table row
 * index[r % n_index] of scale/shift/gate (each addressed with its own row
 * stride). All math is fp32 with one rounding to bf16 at each store.
 * ------------------------------------------------------------------------- */

/* out = RMSNorm(x)*weight*(1+scale[idx])+shift[idx]
 * replaces fused_rmsnorm_modulate  src/h3_flash/runtime/kernels/fusions.py:194
 *          (_rmsnorm_modulate_kernel fusions.py:69-96) */
int h3b_rmsnorm_modulate(void* out, const void* x, const void* weight,
                         const void* scale, const void* shift, const int64_t* index,
                         int64_t rows, int64_t cols, int64_t n_index,
                         int64_t x_row_stride, int64_t out_row_stride,
                         int64_t scale_row_stride, int64_t shift_row_stride,
                         float eps, h3b_stream_t stream);

/* hidden = residual + gate[idx]*branch (stored); normed = RMSNorm(hidden_fp32)*weight*(1+scale)+shift
 * replaces fused_residual_gate_rmsnorm_modulate  fusions.py:218
 *          (_residual_gate_rmsnorm_modulate_kernel fusions.py:23-67) */
int h3b_residual_gate_rmsnorm_modulate(void* hidden_out, void* normed_out,
                                       const void* residual, const void* branch,
                                       const void* weight, const void* gate,
                                       const void* scale, const void* shift,
                                       const int64_t* index, int64_t rows, int64_t cols,
                                       int64_t n_index, int64_t row_stride,
                                       int64_t gate_row_stride, int64_t scale_row_stride,
                                       int64_t shift_row_stride, float eps,
                                       h3b_stream_t stream);

/* out = x*(1+scale[idx])+shift[idx]   (AdaLN modulate without the norm)
 * eager semantics of kernels/transformer.py:72-74 minus norm1; no reference kernel */
int h3b_modulate(void* out, const void* x, const void* scale, const void* shift,
                 const int64_t* index, int64_t rows, int64_t cols, int64_t n_index,
                 int64_t x_row_stride, int64_t out_row_stride, int64_t scale_row_stride,
                 int64_t shift_row_stride, h3b_stream_t stream);

/* out = residual + gate[idx]*branch   (gated residual add)
 * eager semantics of kernels/transformer.py:123-126 (block output); no reference kernel */
int h3b_gated_residual(void* out, const void* residual, const void* branch,
                       const void* gate, const int64_t* index, int64_t rows,
                       int64_t cols, int64_t n_index, int64_t row_stride,
                       int64_t gate_row_stride, h3b_stream_t stream);

/* out[r, :n] = x[r, :n] * silu(x[r, n:2n])
 * replaces fused_swiglu  fusions.py:251 (_swiglu_kernel fusions.py:98-123) */
int h3b_swiglu(void* out, const void* x, int64_t rows, int64_t n,
               int64_t in_row_stride, int64_t out_row_stride, h3b_stream_t stream);

/* out = gelu(x, approximate="tanh") elementwise over rows x cols
 * the FFN activation of the benchmark block (torch.nn.functional.gelu semantics) */
int h3b_gelu_tanh(void* out, const void* x, int64_t rows, int64_t cols,
                  int64_t in_row_stride, int64_t out_row_stride, h3b_stream_t stream);

/* ---------------------------------------------------------------------------
 * Per-head QK RMSNorm + partial rotate-half RoPE, and the packed-Ulysses
 * relayouts.
 * ------------------------------------------------------------------------- */

/* x, out: contiguous [batch, seq, heads, head_dim]; cos/sin fp32 [seq, rotary_dim]
 * (row stride rotary_dim). out = rope(RMSNorm_D(x)*weight) on columns < rotary_dim,
 * RMSNorm_D(x)*weight above.
 * replaces fused_qknorm_rope  fusions.py:268 (_qknorm_partial_rope_kernel fusions.py:125-175) */
int h3b_qknorm_rope(void* out, const void* x, const void* weight, const float* cos,
                    const float* sin, int64_t batch, int64_t seq, int64_t heads,
                    int64_t head_dim, int64_t rotary_dim, float eps,
                    h3b_stream_t stream);

/* Fused QK-norm+RoPE of q and k, plus the destination-major pack of q, k, v:
 * send[dst, row, h, 0:D | D:2D | 2D:3D] = (rope(norm(q)), rope(norm(k)), v)[row, dst*hl+h]
 * with hl = heads/world. q/k/v rows are strided (q_row_stride etc.; heads are
 * contiguous within a row: head stride = head_dim). cos/sin fp32 [rows, rotary_dim].
 * replaces fused_qknorm_rope (x2) + pack_qkv_destination_major
 *          src/h3_flash/runtime/parallel/packed_ulysses.py:178-200, relayout.py:97-130 */
int h3b_qknorm_rope_pack(void* send, const void* q, const void* k, const void* v,
                         int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
                         const void* q_weight, const void* k_weight, const float* cos,
                         const float* sin, int64_t rows, int64_t heads, int64_t head_dim,
                         int64_t rotary_dim, int64_t world, float q_eps, float k_eps,
                         h3b_stream_t stream);

/* The QKV projection with the pack in its epilogue: one tcgen05 GEMM
 * y = x w_qkv^T (+ bias), x [rows, dim] (row stride x_row_stride elements),
 * w_qkv [3*heads*head_dim, dim] (the to_q | to_k | to_v weights stacked, nn.Linear
 * layout), bias [3*heads*head_dim] or NULL; then QK-norm + RoPE of the q and k
 * head rows in fp32 and the destination-major store of q, k, v exactly as
 * h3b_qknorm_rope_pack lays them out (send [world, rows, hl, 3*head_dim]). The
 * projection is not rounded to bf16 before the norm (one rounding, at the store).
 * Needs head_dim 128, an even head count, dim % 64 == 0 and rotary_dim in
 * {0, 64, 96, 128} (else H3B_ERR_UNSUPPORTED). With rotary_dim > 0 the call first
 * relays the RoPE tables into `workspace` (16-byte aligned, at least the bytes
 * h3b_qkv_gemm_pack_workspace_size reports: rows * rotary_dim * 8, caller-owned,
 * only used during the call's kernels) so that the epilogue reads them row-
 * contiguously; a null or short workspace is H3B_ERR_VALUE.
 * replaces to_q/to_k/to_v + fused_qknorm_rope (x2) + pack_qkv_destination_major
 *          packed_ulysses.py:166-200, relayout.py:97-130 */
int h3b_qkv_gemm_pack(void* send, int64_t world, const void* x, int64_t rows, int64_t dim,
                      int64_t x_row_stride, const void* w_qkv, const void* bias,
                      const void* q_weight, const void* k_weight, const float* cos,
                      const float* sin, int64_t heads, int64_t head_dim, int64_t rotary_dim,
                      float q_eps, float k_eps, void* workspace, int64_t workspace_bytes,
                      h3b_stream_t stream);

/* Bytes of workspace h3b_qkv_gemm_pack and h3b_qkv_gemm_pack_p2p need for `rows`
 * local rows (0 without RoPE). Host-only; launches nothing. */
int h3b_qkv_gemm_pack_workspace_size(int64_t rows, int64_t rotary_dim, int64_t* bytes_out);

/* out[row, :n] = act(x W^T + bias): x [rows, dim] (row stride x_row_stride),
 * W [n, dim] row-major (nn.Linear layout), bias [n] or NULL, out row stride
 * out_row_stride; bf16 in/out, fp32 accumulation, one rounding at the store.
 * activation 0: none; 1: GELU-tanh (x * sigmoid(2u), u = sqrt(2/pi)(x +
 * 0.044715 x^3)). Needs dim % 64 == 0 and n % 256 == 0 (else H3B_ERR_UNSUPPORTED).
 * replaces the FFN projection + activation of block.ff  kernels/transformer.py:121-122
 *          (and any plain Linear: to_out, the FFN output projection) */
int h3b_gemm(void* out, int64_t out_row_stride, const void* x, int64_t rows, int64_t dim,
             int64_t x_row_stride, const void* w, int64_t n, const void* bias,
             int64_t activation, h3b_stream_t stream);

/* out[row, :n] = residual[row] + gate[index[row % n_index]] * (x W^T + bias)[row]:
 * the block's closing gated residual fused into the FFN output projection (or any
 * projection followed by a gated residual). residual [rows, n] and the gate table
 * [n_table, n] by row strides; the projection stays in fp32 up to the product.
 * Needs dim % 64 == 0 and n % 256 == 0.
 * replaces output_projection + hidden + gate_mlp[idx] * ffn
 *          kernels/transformer.py:120, :123-126 */
int h3b_gemm_gated_residual(void* out, int64_t out_row_stride, const void* x, int64_t rows,
                            int64_t dim, int64_t x_row_stride, const void* w, int64_t n,
                            const void* bias, const void* residual,
                            int64_t residual_row_stride, const void* gate,
                            int64_t gate_row_stride, const int64_t* index, int64_t n_index,
                            h3b_stream_t stream);

/* out[row, :n_out] = value * silu(gate) of the SwiGLU projection, computed from an
 * interleaved weight: rows [256b, 256b+128) of w_interleaved are value rows
 * [128b, 128b+128) of the projection, rows [256b+128, 256b+256) the gate rows
 * n_out + [128b, 128b+128); bias_interleaved [2 n_out] in the same order, or NULL.
 * The projection stays in fp32 up to the product (one rounding, at the store).
 * Needs dim % 64 == 0 and n_out % 128 == 0.
 * replaces swiglu_layer.proj + fused_swiglu  kernels/transformer.py:112-115,
 *          fusions.py:251-265 */
int h3b_gemm_swiglu(void* out, int64_t out_row_stride, const void* x, int64_t rows,
                    int64_t dim, int64_t x_row_stride, const void* w_interleaved,
                    int64_t n_out, const void* bias_interleaved, h3b_stream_t stream);

/* out[dst, row, h, :] = (q|k|v)[row, dst*hl + h, :], out is [world, rows, hl, 3*head_dim].
 * q/k/v are [rows, heads, head_dim] with element strides (row, head), last dim contiguous.
 * replaces pack_qkv_destination_major  src/h3_flash/runtime/parallel/relayout.py:97-130 */
int h3b_pack_qkv(void* out, const void* q, const void* k, const void* v, int64_t rows,
                 int64_t heads, int64_t head_dim, int64_t world,
                 int64_t q_row_stride, int64_t q_head_stride,
                 int64_t k_row_stride, int64_t k_head_stride,
                 int64_t v_row_stride, int64_t v_head_stride, h3b_stream_t stream);

/* out[row, src, :] = x[src, row, :] for contiguous x [world, rows, inner]
 * replaces merge_heads  src/h3_flash/runtime/parallel/relayout.py:133-159 */
int h3b_merge_heads(void* out, const void* x, int64_t world, int64_t rows,
                    int64_t inner, h3b_stream_t stream);

/* ---------------------------------------------------------------------------
 * Dense non-causal attention, softmax(q k^T * scale) v, bf16 in/out, fp32
 * accumulation; tcgen05 MMA with TMEM accumulators, TMA-fed.
 * q/k/v/out are [batch, seq, heads, head_dim] views given by element strides
 * (batch, row, head); head_dim must be 128 and contiguous; every stride must
 * be a multiple of 8 elements and every base 16-byte aligned.
 * The packed-Ulysses receive buffer [S, hl, 3D] is the view
 *   q = qkv, k = qkv + D, v = qkv + 2D, row stride hl*3D, head stride 3D.
 * Work is split into (batch, head, 256-query-row) units. When the last wave of
 * units would leave SMs idle, those units are split along the keys and merged
 * by a second kernel; that needs `workspace` (16-byte aligned, at least the
 * size h3b_attention_workspace_size reports, caller-owned, only used during the
 * call's kernels). With a null or short workspace every unit runs whole: same
 * results, longer tail.
 * replaces torch SDPA at src/h3_flash/runtime/parallel/packed_ulysses.py:201-209 and
 *          flash_attn_func in src/h3_flash/runtime/attention/dense_fa4.py:74-81, :145
 * ------------------------------------------------------------------------- */
int h3b_attention(void* out, const void* q, const void* k, const void* v,
                  int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads,
                  int64_t head_dim,
                  int64_t q_batch_stride, int64_t q_row_stride, int64_t q_head_stride,
                  int64_t k_batch_stride, int64_t k_row_stride, int64_t k_head_stride,
                  int64_t v_batch_stride, int64_t v_row_stride, int64_t v_head_stride,
                  int64_t o_batch_stride, int64_t o_row_stride, int64_t o_head_stride,
                  float softmax_scale, void* workspace, int64_t workspace_bytes,
                  h3b_stream_t stream);

/* Bytes of workspace h3b_attention can use for this shape on the current
 * device (0 if the shape needs none). Host-only; launches nothing. */
int h3b_attention_workspace_size(int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads,
                                 int64_t head_dim, int64_t* bytes_out);

/* h3b_attention for callers that cannot hand over scratch memory (no reference
 * counterpart: the reference always runs in a framework that allocates). A
 * caller that binds this library over a plain C FFI may own no device
 * allocator, and cudaMalloc on its hot loop would bypass the process's memory
 * pool and can synchronise the device. Here the split-tail workspace is a
 * file-scope 20 MiB device array that every GPU loading the library keeps
 * until exit; shapes needing more return H3B_ERR_VALUE. The first call on a
 * device resolves the array's device address (cudaGetSymbolAddress): make that
 * first call before any stream capture. The address is cached per device and
 * context, so the first call after cudaDeviceReset (a new context) resolves it
 * again; that call too belongs outside a capture. All calls on a device share the
 * array; calls whose kernels overlap on the GPU race, so keep them ordered.
 * Nothing in this path calls cudaMalloc, cudaFree or an allocating library. */
int h3b_attention_noalloc(void* out, const void* q, const void* k, const void* v,
                          int64_t batch, int64_t seq_q, int64_t seq_k, int64_t heads,
                          int64_t head_dim,
                          int64_t q_batch_stride, int64_t q_row_stride, int64_t q_head_stride,
                          int64_t k_batch_stride, int64_t k_row_stride, int64_t k_head_stride,
                          int64_t v_batch_stride, int64_t v_row_stride, int64_t v_head_stride,
                          int64_t o_batch_stride, int64_t o_row_stride, int64_t o_head_stride,
                          float softmax_scale, h3b_stream_t stream);

/* ---------------------------------------------------------------------------
 * Packed-Ulysses exchange over NVLink peer memory. Each rank owns one receive
 * buffer [S_total, hl, 3*head_dim], one merged buffer [rows_local, heads,
 * head_dim] and one flag array of h3b_peer_flags_bytes() zeroed bytes, all in
 * device memory it exports with h3b_ipc_handle; every rank opens the others'
 * with h3b_ipc_open (plain peer mappings). `*_ptrs` arrays are
 * host arrays of `world` device pointers indexed by rank, this rank's own
 * local pointer included; world <= 16. One attention call on every rank runs,
 * on one stream:
 *   h3b_qkv_gemm_pack_p2p (or a projection of its own, then
 *   h3b_qknorm_rope_pack_p2p) -> h3b_peer_barrier -> h3b_attention_p2p on the
 *   own receive buffer -> h3b_peer_barrier
 * (or, unfused, h3b_attention then h3b_scatter_heads_p2p in place of
 * h3b_attention_p2p) and then reads its merged buffer. With that order single
 * buffers are safe across consecutive calls. All ranks must make the same
 * calls in the same order.
 * ------------------------------------------------------------------------- */

/* h3b_qknorm_rope_pack with the pack's store going straight to the owner of
 * each head: row r of this rank (global row row_offset + r) of head
 * g = dst*hl + lh lands at recv_ptrs[dst][((row_offset + r)*hl + lh)*3*head_dim].
 * Needs head_dim 64/128/256, rotary_dim and head_dim - rotary_dim multiples of
 * 16 (else H3B_ERR_UNSUPPORTED).
 * replaces the pack + QKV exchange of _packed_qkv_all_to_all
 *          src/h3_flash/runtime/parallel/packed_ulysses.py:85-108
 *          (pack_qkv_destination_major relayout.py:97-130) */
int h3b_qknorm_rope_pack_p2p(void* const* recv_ptrs, int64_t world, int64_t row_offset,
                             int64_t total_rows, const void* q, const void* k, const void* v,
                             int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
                             const void* q_weight, const void* k_weight, const float* cos,
                             const float* sin, int64_t rows, int64_t heads, int64_t head_dim,
                             int64_t rotary_dim, float q_eps, float k_eps, h3b_stream_t stream);

/* h3b_qkv_gemm_pack with the epilogue storing each head row straight into its
 * owner's receive buffer, at the layout of h3b_qknorm_rope_pack_p2p: the QKV
 * exchange runs inside the GEMM, overlapped with the tiles still computing.
 * Same bits as h3b_qkv_gemm_pack followed by an exchange of its send buffer;
 * workspace as for h3b_qkv_gemm_pack.
 * replaces the QKV projection, the pack and the QKV exchange of
 *          packed_ulysses.py:166-200, :85-108 */
int h3b_qkv_gemm_pack_p2p(void* const* recv_ptrs, int64_t world, int64_t row_offset,
                          int64_t total_rows, const void* x, int64_t rows, int64_t dim,
                          int64_t x_row_stride, const void* w_qkv, const void* bias,
                          const void* q_weight, const void* k_weight, const float* cos,
                          const float* sin, int64_t heads, int64_t head_dim,
                          int64_t rotary_dim, float q_eps, float k_eps, void* workspace,
                          int64_t workspace_bytes, h3b_stream_t stream);

/* out is this rank's attention output [S_total, heads_local, head_dim]
 * (contiguous); global row s, owned by rank o (row_counts[] gives every rank's
 * rows in rank order), goes to
 *   merged_ptrs[o][((s - offset_o)*world + rank)*heads_local*head_dim].
 * replaces _packed_output_all_to_all  packed_ulysses.py:111-128
 *          (exchange + merge_heads relayout.py:133-159) */
int h3b_scatter_heads_p2p(void* const* merged_ptrs, const int64_t* row_counts, const void* out,
                          int64_t world, int64_t rank, int64_t heads_local, int64_t head_dim,
                          h3b_stream_t stream);

/* Attention over this rank's receive buffer qkv = [S_total, heads_local,
 * 3*head_dim] (S_total = sum of row_counts) whose epilogue stores every output
 * row straight into its owner's merged buffer, at the same place
 * h3b_scatter_heads_p2p would put it: the output exchange runs inside the
 * attention kernel, overlapped with the tiles still computing. Results are
 * bit-identical to h3b_attention followed by h3b_scatter_heads_p2p. workspace
 * as for h3b_attention with batch 1, seq_q = seq_k = S_total, heads_local heads.
 * replaces the SDPA call and _packed_output_all_to_all
 *          packed_ulysses.py:201-209, :111-128 (merge_heads relayout.py:133-159) */
int h3b_attention_p2p(void* const* merged_ptrs, const int64_t* row_counts, int64_t world,
                      int64_t rank, const void* qkv, int64_t heads_local, int64_t head_dim,
                      float softmax_scale, void* workspace, int64_t workspace_bytes,
                      h3b_stream_t stream);

/* Cross-rank barrier on the ranks' flag arrays; orders every earlier store of
 * this stream before every later load of the peers' streams. The epoch lives
 * in the flag array, so the call can be captured in a CUDA graph. A peer
 * missing for 10 s sets status bit 2 and the kernel returns.
 * replaces the synchronisation inside dist.all_to_all_single (packed_ulysses.py:67-82) */
int h3b_peer_barrier(void* const* flag_ptrs, int64_t world, int64_t rank, h3b_stream_t stream);
int64_t h3b_peer_flags_bytes(void);

/* CUDA IPC for the buffers above. h3b_ipc_handle writes the 64-byte handle of
 * the allocation holding `ptr` and ptr's offset into it; h3b_ipc_open maps a
 * peer's handle into this process (on the current device) and returns the
 * mapped base + offset; h3b_ipc_close drops it. A handle opened again in the
 * same process shares the first mapping (reference-counted), so buffers carved
 * out of one allocation can be exported separately. No reference counterpart:
 * the reference exchanges through NCCL only. */
#define H3B_IPC_HANDLE_BYTES 64
int h3b_ipc_handle(const void* ptr, void* handle, int64_t* offset);
int h3b_ipc_open(const void* handle, int64_t offset, void** ptr);
int h3b_ipc_close(void* ptr, int64_t offset);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
