/*
 * eraserdit_b200 -- C ABI of the B200 (sm_100a) DiT self-attention hot path.
 *
 * Conventions (the style of the reference's mask-STA ctypes library,
 * layers/attention/backends/mask_sta.py:108-131 and
 * layers/attention/backends/csrc/mask_sta/core.cu:767-788):
 *   - every entry point takes raw device pointers, plain sizes, strides in
 *     ELEMENTS (not bytes) and the caller's CUDA stream (as void*);
 *   - the caller owns every buffer; nothing here allocates device memory;
 *   - work is only enqueued on the given stream; no host synchronisation;
 *   - the return value is 0 on success, a positive cudaError_t from the
 *     launch, or a negative argument error detected before launching
 *     (erd_error_string() describes it);
 *   - `status` pointers (may be NULL) receive device-side error bits: a wait
 *     inside a kernel that timed out (the kernel then returns early instead of
 *     hanging).  The caller reads them after synchronising.
 * BF16 tensors are passed as void* (16-bit words).
 */
#ifndef ERASERDIT_B200_H_
#define ERASERDIT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ERD_ABI_VERSION 5

/* ABI version probe; replaces eraserdit_mask_sta_abi()
 * (layers/attention/backends/csrc/mask_sta/core.cu:767). */
int erd_abi_version(void);

/* Human-readable text for a return code of any entry point. */
const char* erd_error_string(int code);

/*
 * Per-axis RoPE table for the LTX 3D rotary embedding.
 * Replaces the table built by LTXVideoRotaryPosEmbed.forward
 * (models/dits/eraserdit_transformer.py:136-214) in factored form: for axis a
 * in (frame, height, width), coordinate i and frequency k it stores
 * (cos, sin)(freqs[k] * (2 * coord_a(i) - 1)) as float2 at
 * table[2 * (axis_base(a) + i * nfreq + k)], axis_base = 0, F*nfreq,
 * (F+H)*nfreq.  coord_a(i) = i, or, when use_scale != 0,
 * i * scale_a * patch_a / base_a evaluated left to right in fp32 (:153-156).
 * `freqs` are the nfreq = dim/6 base frequencies of :194-201 (device, fp32).
 */
int erd_rope_axis_table(const float* freqs, int nfreq, int frames, int height, int width,
                        int use_scale, float scale_f, float scale_h, float scale_w,
                        float patch_t, float patch_s, float base_f, float base_h, float base_w,
                        float* table, void* stream);

/*
 * Fused QK RMSNorm across heads + 3D RoPE, optionally copying V, writing Q/K/V
 * straight into a head-major destination layout.
 * Replaces apply_fused_qk_rmsnorm_rope
 * (layers/operator_fusion/qk_rmsnorm_rope.py:80-152; semantics of the unfused
 * closure models/dits/eraserdit_attention.py:259-281 with diffusers RMSNorm,
 * rounding boundaries as layers/operator_fusion/triton/rmsnorm_native.py:25-43)
 * and the Ulysses send packing (layers/attention/qkv_packing.py:31-48,
 * models/adapters/eraserdit/nccl_sequence.py:56-65).
 *
 * Inputs: q_in/k_in (and v_in, may be NULL) BF16 [batch][tokens][hidden] with
 * the given token / batch strides; hidden must be 2048 (32 heads x 64).
 * q_weight/k_weight: BF16 [hidden] RMSNorm weights or NULL (no affine).
 * rope_mode 0: no RoPE; 1: full fp32 cos/sin tables indexed
 * [b * tab_batch_stride + t * tab_token_stride + c]; 2: per-axis table from
 * erd_rope_axis_table, token t of this call sitting at grid position
 * token_offset + t of a frames x height x width grid, or, when grid_index
 * (device int32, mode 2 only) is given, at grid_index[token_offset + t]
 * (f * height * width + h * width + w): tokens laid out in another order,
 * such as the tile order of the block-sparse attention.
 * Outputs: element (b, t, head h, d) goes to
 *   out + b*out_batch_stride + t*out_token_stride
 *       + (h % heads_per_dest)*out_head_stride + (h / heads_per_dest)*out_dest_stride + d.
 * Outputs may alias the inputs exactly (in place).
 * With k_in and k_out NULL (rope_mode 0, no V) only Q is normalised: the
 * cross-attention query norm (apply_fused_cross_q_rmsnorm,
 * layers/operator_fusion/cross_q_rmsnorm.py:33-49).
 */
int erd_qk_norm_rope(const void* q_in, const void* k_in, const void* v_in,
                     int64_t in_token_stride, int64_t in_batch_stride, int batch, int tokens,
                     int hidden, const void* q_weight, const void* k_weight, float eps,
                     int rope_mode, const float* cos_tab, const float* sin_tab,
                     int64_t tab_token_stride, int64_t tab_batch_stride, const float* axis_table,
                     int nfreq, int frames, int height, int width, int token_offset,
                     const int32_t* grid_index, void* q_out,
                     void* k_out, void* v_out, int64_t out_token_stride, int64_t out_batch_stride,
                     int64_t out_head_stride, int heads_per_dest, int64_t out_dest_stride,
                     void* stream);

/*
 * Non-causal, unmasked attention, head_dim 64, BF16 in/out, FP32 softmax and
 * accumulation, on tcgen05 tensor cores with TMEM accumulators.
 * Replaces SDPAImpl.forward (layers/attention/backends/sdpa.py:56-80) as
 * called from models/dits/eraserdit_attention.py:287-289 and from the Ulysses
 * path after the sequence-to-head exchange (nccl_sequence.py:259-260).
 *
 * The sequence of every (batch, head) is `nseg` (<= 16) segments held in
 * slots of `seg_len` tokens; segment s holds seg_lens[s] valid tokens
 * (seg_lens: host array of nseg entries, or NULL for all seg_len).  nseg = 1
 * on one GPU; after the Ulysses all-to-all there is one segment per source
 * rank.  Rows past a segment's valid length are never attended to or
 * written; they must hold finite values (e.g. zeros).
 * Element (b, h, segment s, token t, d) of X in {q, k, v} is at
 *   X + s*x_seg_stride + b*x_batch_stride + h*x_head_stride + t*x_token_stride + d,
 * and the output row goes to the same formula with the o_* strides.
 * Pointers must be 16-byte aligned and strides multiples of 8 elements.
 */
int erd_attn_fwd_bf16(const void* q, const void* k, const void* v, int64_t q_token_stride,
                      int64_t q_head_stride, int64_t q_batch_stride, int64_t q_seg_stride,
                      int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
                      int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
                      int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads,
                      int seg_len, int nseg, const int32_t* seg_lens, int head_dim,
                      float softmax_scale, void* out,
                      int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride,
                      int64_t o_seg_stride, int* status, void* stream);

/*
 * Cross-attention, head_dim 64: q_len query tokens against kv_len key/value
 * tokens per (batch, head), BF16 in/out.  kv_valid (host array of `batch`
 * entries, batch <= 16, or NULL for all kv_len) is the attended prefix of the
 * keys of each batch entry: the text padding mask of
 * EraserDiTAttentionProcessor.cross_attn (eraserdit_attention.py:292-332),
 * whose additive -10000 bias (eraserdit_transformer.py:484-487) drives the
 * padded keys' weights to exactly zero in fp32.  Strides as erd_attn_fwd_bf16
 * (one segment).
 */
int erd_attn_fwd_cross_bf16(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
    int64_t v_token_stride, int64_t v_head_stride, int64_t v_batch_stride, int batch, int heads,
    int q_len, int kv_len, const int32_t* kv_valid, int head_dim, float softmax_scale, void* out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride, int* status,
    void* stream);

/*
 * Ring (USP) attention, head_dim 64.  Serves the ring axis of
 * DistributedSequenceRank.attention (models/adapters/eraserdit/nccl_sequence.py:
 * 235-332) and replaces ring_accumulator.piece (layers/attention/
 * ring_accumulator.py:12-100).  The queries are q_nseg segments (q_seg_lens
 * valid tokens each, slots of seg_len tokens) and the keys / values kv_nseg
 * segments (kv_seg_lens valid tokens each, slots of kv_seg_len tokens); the
 * length arrays are host arrays and the strides those of erd_attn_fwd_bf16.
 *   - state_mode 0: one launch over every key segment (the reference's
 *     "reference" ring mode, after its ring gather of K/V shards);
 *   - otherwise one launch per ring piece with a carried softmax state
 *     (the "streaming" mode): bit 1 (read) starts from `state`, bit 2 (write)
 *     stores the state instead of the output.  First piece: 2; middle: 3;
 *     last: 1 (writes the BF16 output).  `state` is caller-owned device
 *     memory, 16-byte aligned, of erd_ring_state_bytes(batch, heads, seg_len,
 *     q_nseg) bytes; it holds O (fp32, unnormalised) and the running max / sum
 *     of every query row.  Pieces of one state run in stream order.
 * seg_out (host array of q_nseg device pointers, or NULL) replaces
 * out + s * o_seg_stride as the output base of query segment s.  out may be
 * NULL when seg_out is given or the state is written.  Returns -6 when
 * state_bytes is too small.
 */
size_t erd_ring_state_bytes(int batch, int heads, int seg_len, int q_nseg);
int erd_attn_fwd_ring_bf16(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int q_nseg,
    const int32_t* q_seg_lens, int kv_seg_len, int kv_nseg, const int32_t* kv_seg_lens,
    int head_dim, float softmax_scale, void* out, int64_t o_token_stride, int64_t o_head_stride,
    int64_t o_batch_stride, int64_t o_seg_stride, void* const* seg_out, void* state,
    size_t state_bytes, int state_mode, int* status, void* stream);

/*
 * Block-sparse variant of erd_attn_fwd_bf16 for the mask-aware pattern.
 * Replaces MaskSTA.__call__ (layers/attention/backends/mask_sta.py:160-194)
 * and its kernel sta_mask_attention (csrc/mask_sta/core.cu); the pattern
 * (mask_sta.py:66-105) arrives as per-CTA work lists instead of the
 * reference's per-query-block LUT:
 *   schedule  device int32 [n_schedule][4], 16-byte aligned: query tile A,
 *             query tile B (or -1), first entry, number of entries (>= 1);
 *   entries   device uint32 [n_entries]: key tile | (64-token halves of the
 *             key tile that A attends, bit 0 = first half) << 24 | (halves B
 *             attends) << 26.
 * Tiles are the 128-token tiles of the segmented layout (segment s, local
 * tile i -> s * ceil(seg_len / 128) + i).  Every query tile to be written
 * appears in exactly one schedule row, with at least one attended half.
 * out_rows (device int32 [seg_len], nseg == 1 only, may be NULL) gives the
 * output token of each query token: the output is scattered back from the
 * tile order the inputs are laid out in.
 * All other arguments and the result are those of erd_attn_fwd_bf16.
 */
int erd_attn_fwd_sparse_bf16(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* out, int64_t o_token_stride,
    int64_t o_head_stride, int64_t o_batch_stride, int64_t o_seg_stride, const int32_t* schedule,
    int n_schedule, const uint32_t* entries, int64_t n_entries, const int32_t* out_rows,
    int* status, void* stream);

/*
 * Token gather: dst[b][t][:] = src[b][index[t]][:] for rows of row_elems
 * BF16 values (a multiple of 8), index a device int32 [tokens] with entries
 * in [0, src_tokens).  Lays Q/K/V out in the tile order of the block-sparse
 * pattern, replacing the row_order gathers of the reference's quantisation
 * kernels (layers/attention/backends/mask_sta.py:28-63) and V preparation
 * (sta_mask_prepare_v).  Strides in elements, multiples of 8.
 */
int erd_gather_tokens(const void* src, int64_t src_token_stride, int64_t src_batch_stride,
                      int src_tokens, void* dst, int64_t dst_token_stride,
                      int64_t dst_batch_stride, const int32_t* index, int batch, int tokens,
                      int row_elems, void* stream);

/*
 * erd_qk_norm_rope with every head group stored straight into another rank's
 * receive buffer (the input all-to-all of Ulysses SP as peer stores over
 * NVLink).  Replaces pack_qkv + the first all_to_all_single of
 * DistributedSequenceRank._ulysses_input (nccl_sequence.py:43-79,
 * communication_op.py:97-137).  Head group g = head / heads_per_dest goes to
 * dest_bases[g] (ndest device pointers, CUDA IPC mappings of the peers'
 * buffers or local memory): Q at +0, K at +k_offset, V at +v_offset elements,
 * element (b, t, head, d) at + b*out_batch_stride + t*out_token_stride
 * + (head % heads_per_dest)*out_head_stride + d.  Other arguments as
 * erd_qk_norm_rope.
 */
int erd_qk_norm_rope_peer(const void* q_in, const void* k_in, const void* v_in,
                          int64_t in_token_stride, int64_t in_batch_stride, int batch, int tokens,
                          int hidden, const void* q_weight, const void* k_weight, float eps,
                          int rope_mode, const float* cos_tab, const float* sin_tab,
                          int64_t tab_token_stride, int64_t tab_batch_stride,
                          const float* axis_table, int nfreq, int frames, int height, int width,
                          int token_offset, const int32_t* grid_index, void* const* dest_bases,
                          int ndest, int64_t k_offset, int64_t v_offset, int64_t out_token_stride,
                          int64_t out_batch_stride, int64_t out_head_stride, int heads_per_dest,
                          void* stream);

/*
 * erd_attn_fwd_bf16 with the output rows of segment s stored at seg_out[s]
 * (nseg device pointers: the token owners' return buffers, peer or local) +
 * b*o_batch_stride + h*o_head_stride + t*o_token_stride.  Replaces the second
 * all-to-all (DistributedSequenceRank._ulysses_output, nccl_sequence.py:81-103).
 */
int erd_attn_fwd_bf16_peer(const void* q, const void* k, const void* v, int64_t q_token_stride,
                           int64_t q_head_stride, int64_t q_batch_stride, int64_t q_seg_stride,
                           int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
                           int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
                           int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads,
                           int seg_len, int nseg, const int32_t* seg_lens, int head_dim,
                           float softmax_scale, void* const* seg_out, int64_t o_token_stride,
                           int64_t o_head_stride, int64_t o_batch_stride, int* status,
                           void* stream);

/*
 * The block-sparse and FP8 attentions with the same per-segment output
 * pointers (erd_attn_fwd_sparse_bf16 / erd_attn_fwd_fp8 arguments otherwise;
 * out and o_seg_stride replaced by seg_out).
 */
int erd_attn_fwd_sparse_bf16_peer(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* const* seg_out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride,
    const int32_t* schedule, int n_schedule, const uint32_t* entries, int64_t n_entries,
    int* status, void* stream);

int erd_attn_fwd_fp8_peer(const void* q, const void* k, const void* v, int64_t q_token_stride,
                          int64_t q_head_stride, int64_t q_batch_stride, int64_t q_seg_stride,
                          int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
                          int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
                          int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads,
                          int seg_len, int nseg, const int32_t* seg_lens, int head_dim,
                          float softmax_scale, void* const* seg_out, int64_t o_token_stride,
                          int64_t o_head_stride, int64_t o_batch_stride, void* workspace,
                          size_t workspace_bytes, int* status, void* stream);

/*
 * Peer-exchange plumbing (no counterpart entry in the reference, whose
 * exchange is NCCL's).  erd_peer_alloc is the one allocating entry point: it
 * cudaMallocs (and zeroes) a buffer that peers map with the 64-byte handle of
 * erd_peer_ipc_handle / erd_peer_ipc_open (cudaIpcMemLazyEnablePeerAccess).
 * erd_peer_signal: after the stream's earlier stores, a system-scope fence and
 * a release store of `epoch` to each of the npeers flag slots (device
 * pointers, this rank's slot in every rank's flag array).  erd_peer_wait:
 * acquire loads of n local flags until each equals `epoch`, at most
 * timeout_ns; on timeout the status word gets 0x10 and the kernel returns.  A
 * rank whose phase failed signals -epoch: waiters then set 0x20 and return.
 */
int erd_peer_alloc(size_t bytes, void** ptr);
int erd_peer_free(void* ptr);
int erd_peer_ipc_handle(void* ptr, void* handle64);
int erd_peer_ipc_open(const void* handle64, void** ptr);
int erd_peer_ipc_close(void* ptr);
int erd_peer_signal(int32_t* const* peer_slots, int npeers, int32_t epoch, void* stream);
int erd_peer_wait(const int32_t* flags, int n, int32_t epoch, int64_t timeout_ns, int* status,
                  void* stream);

/*
 * Static-scale E4M3 quantisation of n BF16 values (n a multiple of 16):
 * out[i] = E4M3_RN(clamp(x[i] / scale, -448, 448)) with an IEEE division.
 * Replaces the activation quantiser of SharedQKV
 * (layers/quantization/qkv_fp8.py:52-55; _quant_fp8_tensor,
 * layers/quantization/eraserdit_fp8.py:60-69).
 */
int erd_quantize_e4m3(const void* x, void* out, int64_t n, float scale, void* stream);

/*
 * Linear layer y = x W^T + b with BF16 operands, FP32 accumulation, the bias
 * added in FP32 and one rounding to BF16 (the semantics of torch's
 * F.linear(x, W, b) for BF16 tensors): x [m, k] with row stride ldx, W [n, k]
 * (nn.Linear's weight layout) with row stride ldw, bias [n] or NULL, y [m, n]
 * with row stride ldy, strides in elements.  n must be a multiple of 256, k a
 * multiple of 64; pointers and strides 16-byte aligned.
 * Replaces the nn.Linear products of the self-attention path: the Q/K/V
 * projections attn.to_q/to_k/to_v (models/dits/eraserdit_attention.py:248-253,
 * run as one product over the concatenated weights) and the output projection
 * to_out[0] (models/dits/eraserdit_attention.py:216-229).
 */
int erd_linear_bf16(const void* x, int64_t ldx, const void* weight, int64_t ldw, const void* bias,
                    void* y, int64_t ldy, int m, int n, int k, int* status, void* stream);

/*
 * erd_linear_bf16 with the columns from scatter_col0 on stored into other
 * buffers instead of y: column j >= scatter_col0 of row i goes to
 * dest_bases[g], g = (j - scatter_col0) / group_cols, at element offset
 * (i / rows_per_batch) * dest_batch_stride + (i % rows_per_batch) *
 * dest_token_stride + (j - scatter_col0) % group_cols.  Columns below
 * scatter_col0 go to y as in erd_linear_bf16.  scatter_col0 a multiple of 256,
 * group_cols a power of two >= 128, ndest * group_cols == n - scatter_col0
 * (at most 16 destinations), m a multiple of rows_per_batch, destinations and
 * strides 16-byte aligned.
 * On the Ulysses peer path this stores V (columns 4096..6143 of the
 * concatenated projection) straight into every rank's receive slot over
 * NVLink, in the layout of the seq->head all-to-all that follows the
 * projection (layers/attention/qkv_packing.py:31-48, nccl_sequence.py:43-79):
 * the projection's epilogue carries V's exchange, and the prologue only Q, K.
 */
int erd_linear_bf16_scatter(const void* x, int64_t ldx, const void* weight, int64_t ldw,
                            const void* bias, void* y, int64_t ldy, int m, int n, int k,
                            int scatter_col0, void* const* dest_bases, int ndest, int group_cols,
                            int rows_per_batch, int64_t dest_batch_stride,
                            int64_t dest_token_stride, int* status, void* stream);

/*
 * The same product with E4M3 operands (one byte each):
 * y = BF16(acc * col_scale[j] + bias[j]) with acc the FP32 sum of x[i, :] *
 * W[j, :]; col_scale [n] FP32 (activation scale times the weight scale of the
 * column's projection), bias [n] BF16 or NULL.  n a multiple of 256, k a
 * multiple of 128; strides in elements, rows 16-byte aligned.
 * Replaces the scaled_mm products of SharedQKV (layers/quantization/qkv_fp8.py:
 * 29-63: x_fp8 @ w_fp8^T with scale_a, scale_b, bias, BF16 out), as one
 * product over the concatenated Q/K/V weights.
 */
int erd_linear_fp8(const void* x, int64_t ldx, const void* weight, int64_t ldw,
                   const float* col_scale, const void* bias, void* y, int64_t ldy, int m, int n,
                   int k, int* status, void* stream);

/*
 * SageAttention-style FP8 attention, head_dim 64: K smoothed by its per-head
 * token mean, Q and K quantised to E4M3 per 128-token block, V to E4M3 per
 * channel, P to E4M3 (scaled by 448), FP32 accumulation (tcgen05
 * kind::f8f6f4).  Replaces SageFP8AttentionImpl.forward
 * (layers/attention/backends/sage_fp8.py:174-219) with its peripheral
 * quantization (layers/attention/backends/sage_peripheral.py:33-81).
 * Inputs, sequence segments and output use exactly the addressing of
 * erd_attn_fwd_bf16.  `workspace` (1024-byte aligned, at least
 * erd_attn_fp8_workspace_bytes(...) bytes, caller-owned) receives the
 * quantised operands and scales; the call does not allocate.
 */
size_t erd_attn_fp8_workspace_bytes(int batch, int heads, int seg_len, int nseg);

int erd_attn_fwd_fp8(const void* q, const void* k, const void* v, int64_t q_token_stride,
                     int64_t q_head_stride, int64_t q_batch_stride, int64_t q_seg_stride,
                     int64_t k_token_stride, int64_t k_head_stride, int64_t k_batch_stride,
                     int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
                     int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads,
                     int seg_len, int nseg, const int32_t* seg_lens, int head_dim,
                     float softmax_scale, void* out, int64_t o_token_stride,
                     int64_t o_head_stride, int64_t o_batch_stride, int64_t o_seg_stride,
                     void* workspace, size_t workspace_bytes, int* status, void* stream);

/*
 * erd_attn_fwd_fp8 without a caller workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they run attention (a host on the plain C ABI without a caching allocator,
 * where each cudaMalloc would synchronise the device, or a server whose HBM
 * budget is fixed at start-up).  The workspace is a static device array of
 * the library; the call allocates nothing.
 *   - Shapes needing more than ERD_FP8_STATIC_SCRATCH_BYTES of workspace
 *     (erd_attn_fp8_workspace_bytes) return -6 before anything is enqueued.
 *   - The first call on a device looks up the array's address with that
 *     device current; make it before any stream capture.
 *   - All calls on a device share the array: calls that may overlap in time
 *     (other streams, unordered host threads) race on it.
 *   - Nothing in the array needs to start at zero.
 * Arguments and results are those of erd_attn_fwd_fp8.
 */
#define ERD_FP8_STATIC_SCRATCH_BYTES ((size_t)64 << 20)

int erd_attn_fwd_fp8_static_scratch(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride, int64_t o_seg_stride,
    int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ERASERDIT_B200_H_ */
