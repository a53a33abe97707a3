/*
 * fastdecisions-b200 C ABI: the drop-in boundary for the forward hot path of the FastDecisions
 * one-pass decision model (a Qwen3.5-style hybrid decoder: Gated-DeltaNet linear-attention layers
 * and gated GQA attention layers), built for NVIDIA B200 (sm_100a).
 *
 * Conventions (all entry points):
 *   - Plain device pointers, element counts and strides (in elements), no framework types.
 *   - Tensors are bf16 (__nv_bfloat16 bit patterns) unless a parameter says float32/int32.
 *   - `stream` is a cudaStream_t (may be NULL for the legacy default stream).  Every entry point
 *     only enqueues work: no allocation, no host synchronisation, a fixed launch configuration for
 *     a given shape, so calls can be captured into CUDA graphs.
 *   - Return value: FDK_OK (0) or one of the FDK_ERR_* codes below; fdk_get_last_error_string()
 *     then describes the failure (thread-local).  The library never aborts the process.
 *   - The library never allocates device memory.  Scratch space, where an op needs it, is passed
 *     in by the caller (see fdk_chunk_gated_delta_rule_workspace_size).
 *
 * Reference interfaces each entry point replaces are cited as file:line of the FastDecisions
 * repository (src/decider/...) or of transformers 5.5.0 models/qwen3_5/modeling_qwen3_5.py
 * (written [tf]:line), which holds the model arithmetic the reference calls.
 */
#ifndef FASTDECISIONS_B200_FDK_H_
#define FASTDECISIONS_B200_FDK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FDK_OK 0
#define FDK_ERR_INVALID_ARGUMENT 1 /* bad shape, size, null pointer or stride                  */
#define FDK_ERR_ALIGNMENT 2        /* a pointer or stride breaks the 16-byte alignment rule       */
#define FDK_ERR_UNSUPPORTED 3      /* valid request outside what the kernels implement           */
#define FDK_ERR_LAUNCH 4           /* the CUDA launch itself failed                               */
#define FDK_ERR_DEVICE 5           /* no CUDA device, or the device is not sm_100               */

/* Library version string, e.g. "fastdecisions-b200 0.1.0 sm_100a". */
const char* fdk_version(void);

/* Message for the last non-zero status returned on this host thread. */
const char* fdk_get_last_error_string(void);

/*
 * Fused residual add + Qwen3.5 RMSNorm (one row per 128-thread warp group).
 * Replaces `fastdecisions::residual_rms(a, b, weight)` (src/decider/persistent_residual_rms.py:7-14,
 * launcher persistent_residual_rms_kernel.py:75-104) with the eager semantics of
 * [tf]:711-728 + [tf]:775-779:
 *     s   = bf16(x + residual)                 (s = x when residual == NULL)
 *     out = bf16(s * rsqrt(mean(s^2) + eps) * (weight_offset + w))
 * and also writes s to residual_out when it is non-NULL (the reference kernel omits eps and
 * never writes s).  With residual_is_fp32 != 0 the residual stream (residual and residual_out)
 * is float32 and s is not rounded (s = x + residual in fp32).  x and out are bf16; weight is
 * bf16, or float32 when weight_is_fp32 != 0.  Row strides ld_* are in elements and must keep
 * every row 16-byte aligned; hidden % 8 == 0, hidden <= 8192.  residual_out may alias residual.
 * x may be NULL when residual is given: s = residual (the norm of a residual stream whose
 * producer already added into it, as fdk_gemm_bf16_residual_add does).
 */
int fdk_residual_rmsnorm(const void* x, int64_t ld_x, const void* residual, int64_t ld_residual,
                         int residual_is_fp32, const void* weight, int weight_is_fp32, void* out,
                         int64_t ld_out, void* residual_out, int64_t ld_residual_out, int64_t rows,
                         int64_t hidden, float eps, float weight_offset, void* stream);

/*
 * Packed depthwise causal conv1d (width kernel_width <= 4, zero left padding) + SiLU that writes
 * q, k, v directly in the [B, T, H, D] layout the delta rule reads.
 * Replaces `fastdecisions::packed_conv(x, weight)` (src/decider/packed_conv.py:12-21, launcher
 * packed_conv_kernel.py:194-232 `prep_qkv`), generalised from T=2048/C=6144 to any T and
 * C = 2*key_dim + value_dim, plus packed varlen input:
 *     x: [batch, seqlen, C] with row stride ld_x; weight: [C, kernel_width] bf16 contiguous
 *     cu_seqlens: NULL (dense batch) or int32 [num_segments + 1] device array over the flattened
 *                 tokens (batch must be 1); each segment starts with a zero history.
 *     q, k: [batch*seqlen, key_dim], v: [batch*seqlen, value_dim], contiguous.
 */
int fdk_packed_conv_silu(const void* x, int64_t ld_x, const void* weight, int64_t batch,
                         int64_t seqlen, int64_t channels, int kernel_width,
                         const int32_t* cu_seqlens, int64_t num_segments, int64_t key_dim,
                         int64_t value_dim, void* q, void* k, void* v, void* stream);

/*
 * Gated-DeltaNet gate transform:  g = -exp(A_log) * softplus(a + dt_bias)  (float32 out),
 * beta = sigmoid(b) (bf16 out).  Replaces `fastdecisions::unpack_gate` (src/decider/
 * combined_gates.py:6-16, kernel unpack_gate_transform_kernel.py:52-89) and [tf]:491-493.
 * a, b: [tokens, heads] with row strides ld_a, ld_b (elements); A_log, dt_bias: float32 [heads].
 * g: float32 [tokens, heads]; beta: bf16 [tokens, heads], contiguous.
 */
int fdk_gdn_gates(const void* a, int64_t ld_a, const void* b, int64_t ld_b, const float* A_log,
                  const float* dt_bias, float* g, void* beta, int64_t tokens, int64_t heads,
                  void* stream);

/*
 * Scratch bytes fdk_chunk_gated_delta_rule_fwd needs for `tokens` packed tokens split into
 * `num_segments` sequences with `heads` heads of key dim dk and value dim dv.
 */
size_t fdk_chunk_gated_delta_rule_workspace_size(int64_t tokens, int64_t num_segments,
                                                 int64_t heads, int64_t dk, int64_t dv);

/*
 * Chunked gated delta rule (chunk 64), the linear-attention core of the GDN layer.
 * Replaces transformers' `torch_chunk_gated_delta_rule` / fla `chunk_gated_delta_rule`
 * ([tf]:234-311, called at [tf]:499-508 and src/decider/packed_conv.py:55-59) with
 * use_qk_l2norm_in_kernel=True semantics:
 *     q, k: [tokens, heads, dk] bf16 (row stride ld_qk elements per token);
 *     v: [tokens, heads, dv] bf16 (row stride ld_v);
 *     g: float32 [tokens, heads] (per-token log decay), beta: bf16 [tokens, heads];
 *     cu_seqlens: int32 [num_segments + 1] device array (tokens = cu_seqlens[num_segments]);
 *     initial_state: NULL or float32 [num_segments, heads, dk, dv];
 *     out: [tokens, heads, dv] bf16 contiguous; final_state: NULL or float32
 *          [num_segments, heads, dk, dv];
 *     workspace: caller-owned device scratch of at least
 *                fdk_chunk_gated_delta_rule_workspace_size(...) bytes, 256-byte aligned.
 * Supports dk == dv == 128.  Internally fp32 for the l2 norms, the decay cumsum, the
 * unit-lower-triangular solve and the recurrent state; bf16 tensor-core products with fp32
 * accumulation for the chunk matmuls.
 */
int fdk_chunk_gated_delta_rule_fwd(const void* q, const void* k, int64_t ld_qk, const void* v,
                                   int64_t ld_v, const float* g, const void* beta,
                                   const int32_t* cu_seqlens, int64_t num_segments,
                                   int64_t tokens, int64_t heads, int64_t dk, int64_t dv,
                                   float scale, const float* initial_state, void* out,
                                   float* final_state, void* workspace, size_t workspace_bytes,
                                   void* stream);

/*
 * The Gated-DeltaNet mixer core from the projection: packed causal conv (width 4) + SiLU of the
 * projection's q / k / v columns, the gates g = -exp(A_log) softplus(a + dt_bias) and
 * beta = sigmoid(b) from its a / b columns, and the chunked delta rule -- one call, without the
 * [T, H, 128] q / k / v and [T, H] g / beta round trips through HBM.
 * Replaces the sequence the reference's linear-attention forward runs on the projection
 * ([tf]:468-496 of transformers' modeling_qwen3_5.py: causal_conv1d_fn, the gate transform of
 * src/decider/unpack_gate_transform_kernel.py:52-89, chunk_gated_delta_rule); its results are
 * those of fdk_packed_conv_silu, fdk_gdn_gates and fdk_chunk_gated_delta_rule_fwd in sequence
 * (same arithmetic and bf16 roundings).
 *   proj        [tokens, ld_proj] bf16: columns [0, key_dim) q, [key_dim, 2 key_dim) k,
 *               [2 key_dim, 2 key_dim + value_dim) v, a_col + h and b_col + h the gates' a and b
 *   conv_weight [2 key_dim + value_dim, kernel_width] bf16 (kernel_width 4)
 *   A_log, dt_bias [heads] fp32; key_dim = value_dim = heads x 128
 *   workspace   as fdk_chunk_gated_delta_rule_fwd (same size function)
 */
int fdk_gdn_fused_delta_rule_fwd(const void* proj, int64_t ld_proj, const void* conv_weight,
                                 int kernel_width, int64_t key_dim, int64_t value_dim,
                                 int64_t a_col, int64_t b_col, const float* A_log,
                                 const float* dt_bias, const int32_t* cu_seqlens,
                                 int64_t num_segments, int64_t tokens, int64_t heads, float scale,
                                 const float* initial_state, void* out, float* final_state,
                                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * Allocation-free form of fdk_chunk_gated_delta_rule_fwd (same arguments and results, no
 * workspace).  No counterpart in the reference.  It is for callers that cannot allocate device
 * memory: programs that reach this library only through its C ABI and own no device allocator
 * (a cgo, JNI or ctypes host without a CUDA framework), and servers that must not call
 * cudaMalloc / cudaFree on the request path because those calls synchronise the device.
 *   - Scratch: a 32 MiB array inside the library (one per GPU that loads it, held until the
 *     process exits).  A call whose fdk_chunk_gated_delta_rule_workspace_size(...) exceeds
 *     32 MiB is rejected with FDK_ERR_UNSUPPORTED before anything is launched (one 1536-token
 *     request with 16 heads needs about 29.5 MiB).
 *   - The first call on a device looks up the array's device address there (with that device
 *     current) and caches it; make that first call before any stream capture.  The cache
 *     outlives cudaDeviceReset: after a reset of a device this entry point must not be used
 *     on it again in the same process.
 *   - Nothing in the scratch has to start at zero: each call rebuilds its chunk table and every
 *     tile it reads.  All calls on a device share the one array and it keeps the last call's
 *     contents, so calls that overlap on the GPU (concurrent streams) race; serialise them.
 *   - It calls no cudaMalloc, cudaFree or allocating library routine.
 */
int fdk_chunk_gated_delta_rule_fwd_noalloc(const void* q, const void* k, int64_t ld_qk,
                                           const void* v, int64_t ld_v, const float* g,
                                           const void* beta, const int32_t* cu_seqlens,
                                           int64_t num_segments, int64_t tokens, int64_t heads,
                                           int64_t dk, int64_t dv, float scale,
                                           const float* initial_state, void* out,
                                           float* final_state, void* stream);

/*
 * Gated RMSNorm of the GDN output, per head row of width dv:
 *     out = bf16(w * (o * rsqrt(mean(o^2) + eps)) * silu(z))
 * Replaces Qwen3_5RMSNormGated / fla FusedRMSNormGated ([tf]:175-190, call site [tf]:526-529).
 * o: [tokens, heads, dv] contiguous; z: [tokens, heads*dv] with row stride ld_z;
 * weight: [dv] bf16 (weight_is_fp32 = 0) or float32; out: [tokens, heads*dv] contiguous.
 */
int fdk_gated_rmsnorm(const void* o, const void* z, int64_t ld_z, const void* weight,
                      int weight_is_fp32, void* out, int64_t tokens, int64_t heads, int64_t dv,
                      float eps, void* stream);

/*
 * Attention-layer prologue: q_norm / k_norm (Qwen3.5 RMSNorm with 1+w over head_dim) and partial
 * rotary embedding of the first rot_dim features ([tf]:657-668; patched form
 * experiments/native_gqa/bench_native_gqa_model.py:43-53).
 *     qkv: [tokens, ld_qkv] projection output laid out as q_proj ([hq, 2, head_dim]: query then
 *          output gate per head) followed by k_proj [hkv, head_dim] (v_proj after it is untouched)
 *     positions: int32 [tokens] (position within the request, 0 <= pos < max_pos);
 *     rope_table: float32 [max_pos, rot_dim]: row p holds cos(p * inv_freq[i]) for i < rot_dim/2
 *                 then sin(p * inv_freq[i]) ([tf]:139-155 computes the same table in float32);
 *     q_out: [tokens, hq, head_dim], k_out: [tokens, hkv, head_dim] contiguous.
 * Supports head_dim == 128 or 256 and rot_dim <= head_dim, rot_dim % 8 == 0.
 */
int fdk_attn_qk_norm_rope(const void* qkv, int64_t ld_qkv, const void* q_norm_w,
                          const void* k_norm_w, int weight_is_fp32, const int32_t* positions,
                          const float* rope_table, int64_t max_pos, int rot_dim, void* q_out,
                          void* k_out, int64_t tokens, int64_t hq, int64_t hkv, int64_t head_dim,
                          float eps, void* stream);

/*
 * Native GQA causal attention, tcgen05 tensor cores with TMEM accumulators fed by TMA.
 * Replaces `native_gqa_attention(q, k, v)` (src/decider/native_gqa_kernel.py:116-173) and the
 * SDPA path with repeat_kv ([tf]:582-617): query head h reads KV head h / (hq / hkv) directly.
 *     q: [tokens, hq, head_dim] (token stride ld_q elements, head stride head_dim);
 *     k, v: [tokens, hkv, head_dim] (token strides ld_k, ld_v);
 *     cu_seqlens: int32 [num_segments + 1] device array (packed varlen; causal inside each
 *                 segment, no attention across segments); max_seqlen bounds the longest segment;
 *     gate: NULL, or [tokens, hq*head_dim] with row stride ld_gate (and head stride 2*head_dim
 *           when gate_interleaved != 0): out = attn * sigmoid(gate) ([tf]:687-689) fused;
 *     out: [tokens, hq, head_dim] contiguous bf16.
 * Softmax statistics are float32 (online, exp2 domain); P is rounded to bf16 before P.V.
 * Supports head_dim == 128; all strides must be multiples of 8 elements (16-byte TMA rule).
 */
int fdk_gqa_fwd(const void* q, int64_t ld_q, const void* k, int64_t ld_k, const void* v,
                int64_t ld_v, const int32_t* cu_seqlens, int64_t num_segments,
                int64_t max_seqlen, int64_t tokens, int64_t hq, int64_t hkv, int64_t head_dim,
                float scale, const void* gate, int64_t ld_gate, int gate_interleaved, void* out,
                void* stream);

/*
 * Reads and clears the device-side error word of the current device.  Kernels that wait on
 * mbarriers (fdk_gqa_fwd, the delta rule) bound every wait; a wait that runs out sets a bit of
 * this word, frees its resources and returns without finishing its tile.  Bits: 1 an attention
 * wait ran out, 2 a delta-rule wait ran out, 4 the bounded-wait self-test, 8 the delta rule found
 * cu_seqlens invalid on the device (cu[0] != 0, decreasing, or cu[num_segments] != tokens) and
 * treated every segment as empty, 16 a GEMM wait ran out.  Synchronises with the device.
 * No reference counterpart (the reference's Triton kernels have no device waits).
 */
int fdk_poll_device_error(int* code);

/*
 * Self-test of that failure path, with no GPU fault: one warp waits on an mbarrier that nothing
 * arrives on, through the bounded wait the kernels use; after `budget_cycles` SM clock cycles
 * (at most 4e9) the wait gives up, bit 2 (value 4) of the device error word is set and the
 * kernel returns.  The context stays usable.  No reference counterpart.
 */
int fdk_selftest_bounded_wait(int64_t budget_cycles, void* stream);

/*
 * Projection / MLP GEMM on the tcgen05 tensor cores: C = A B^T, bf16 inputs, fp32 accumulation.
 * Replaces the nn.Linear GEMMs of the layer ([tf]:442-449, 532, 657-664, 691, 706-708; the
 * reference's engine runs them as cuBLAS through torch) with the epilogue fused:
 *     A [m, k] (row stride lda), B [n, k] (row stride ldb): the weight in nn.Linear layout;
 *     epilogue 0: C [m, n] = bf16(A B^T)                         (row stride ldc)
 *     epilogue 1: SwiGLU, [tf]:706-708.  B holds gate_proj and up_proj rows interleaved in blocks
 *                 of 128 (block j: gate rows 128 j .. 128 j + 127, then the same up rows), n = 2 I
 *                 a multiple of 256; C [m, I] = bf16(silu(A gate^T) * (A up^T)) computed from the
 *                 fp32 accumulators (the [m, 2 I] projection is never stored).
 * n and k multiples of 8, every pointer and row stride 16-byte aligned; ragged m, n, k are handled.
 */
int fdk_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc,
                  int64_t m, int64_t n, int64_t k, int epilogue, void* stream);

/*
 * The attention layer's projection GEMM with its prologue ops fused into the epilogue: C = A B^T
 * as fdk_gemm_bf16 (B = [q_proj; k_proj; v_proj] weights, q_proj rows laid out per head as the
 * query then the output gate, [tf]:657-659), and for every query and key head block of the result:
 * RMSNorm with (1 + w) over the head ([tf]:662-663) and the rotary embedding of its first
 * rot_dim = head_dim / 4 features ([tf]:666-667), computed from the fp32 accumulators, written to
 * q_out [m, hq, head_dim] and k_out [m, hkv, head_dim] (contiguous).  C [m, n] (row stride ldc)
 * receives the output-gate and v columns; its q and k columns are not written.  Replaces the
 * GEMM + fdk_attn_qk_norm_rope pair (same arithmetic, without rounding q / k to bf16 before the
 * norm).  n = (2 hq + 2 hkv) head_dim; head_dim 128 or 256; positions, rope_table and max_pos as
 * fdk_attn_qk_norm_rope; norm weights bf16 [head_dim].
 */
int fdk_gemm_bf16_qk_norm_rope(const void* a, int64_t lda, const void* b, int64_t ldb, void* c,
                               int64_t ldc, int64_t m, int64_t n, int64_t k, int64_t hq,
                               int64_t hkv, int64_t head_dim, const void* q_norm_w,
                               const void* k_norm_w, const int32_t* positions,
                               const float* rope_table, int64_t max_pos, int rot_dim, float eps,
                               void* q_out, void* k_out, void* stream);

/*
 * Projection GEMM that adds into the residual stream: h [m, n] (float32, row stride ldh) += A B^T,
 * the residual adds of the decoder layer ([tf]:775 and 781) fused into the out-projection and
 * down-projection GEMMs that produce them ([tf]:532, 691, 708).  The fp32 accumulators are added
 * into h by TMA reduce-add stores: the layer output is never rounded to bf16, and K can be split
 * into slices that each add their partial sum (split_k: 1-16 slices; 0 = 1: measured, ordered
 * slices cost more than the idle SMs they fill at m = 1536, n = 2048).
 * The slices of a tile add in a fixed order (slice 0 first), so results are reproducible; the
 * order is kept with `tickets`: int32 [4 x ceil(m / 128) x ceil(n / 256) + 2], zero before the
 * first call and left zero by every call that completes (re-zero it after an error of this call).
 * With split slices the CTAs claim work dynamically, so the call stays deadlock-free when other
 * kernels hold some of the SMs.
 * tickets == NULL runs without splitting.  n and k multiples of 8; pointers and rows 16-byte
 * aligned (ldh a multiple of 4).  Calls sharing one tickets array must not overlap on the GPU.
 */
int fdk_gemm_bf16_residual_add(const void* a, int64_t lda, const void* b, int64_t ldb, float* h,
                               int64_t ldh, int64_t m, int64_t n, int64_t k, int split_k,
                               int32_t* tickets, void* stream);

/*
 * Projection GEMM split along K into `slices` parts whose fp32 products land in separate planes:
 * partials [slices][m][n] (contiguous float32), plane s = A[:, K_s] B[:, K_s]^T over the s-th
 * slice of K.  For the out / down projections at batch-1 sizes, where the output tiles alone leave
 * SMs idle (m = 1536, n = 2048: 96 tiles for 148 SMs); fdk_rmsnorm_add_partials then adds the
 * planes into the residual stream in a fixed order ([tf]:775, 781), so results are reproducible and
 * the layer output is never rounded to bf16 (measured: in the config-4 forward this pair is
 * slower than a cuBLAS GEMM + fdk_residual_rmsnorm, 5.77 vs 5.30 ms).  Every slice must be non-empty
 * (slices <= ceil(k / 64), and no slice left empty by rounding); n and k multiples of 8.
 */
int fdk_gemm_bf16_partials(const void* a, int64_t lda, const void* b, int64_t ldb, float* partials,
                           int64_t m, int64_t n, int64_t k, int slices, void* stream);

/*
 * h [rows, hidden] (float32) += partials[0] + ... + partials[nparts - 1] (planes of
 * [rows][hidden] float32, added in that order), then out = bf16(h * rsqrt(mean(h^2) + eps) *
 * (weight_offset + w)) when out is non-NULL ([tf]:711-728 after the residual add of [tf]:775 /
 * 781).  hidden a multiple of 8, at most 4096.
 */
int fdk_rmsnorm_add_partials(const float* partials, int nparts, float* h, int64_t ldh,
                             const void* weight, int weight_is_fp32, void* out, int64_t ld_out,
                             int64_t rows, int64_t hidden, float eps, float weight_offset,
                             void* stream);

/* Token embedding gather: out[t, :] = table[ids[t], :] ([tf]:1243).  ids int32. */
int fdk_embed(const int32_t* ids, const void* table, int64_t vocab, int64_t hidden, void* out,
              int64_t tokens, void* stream);

/* SwiGLU: out[t, i] = bf16(silu(gu[t, i]) * gu[t, inter + i]) ([tf]:706-708); gu row stride
 * ld_gu (elements), out [tokens, inter] contiguous. */
int fdk_swiglu(const void* gu, int64_t ld_gu, void* out, int64_t tokens, int64_t inter,
               void* stream);

/*
 * Slot readout: final RMSNorm (1+w) of the slot rows, restricted logits over `num_letters`
 * candidate rows and a masked, temperature-scaled softmax.  Replaces the slot gather,
 * F.linear(h, W_letters) and read_slots/scaled_softmax of src/decider/model.py:18-27 and
 * src/decider/engine.py:48-56 (temperature.py:136-144).
 *     hidden: [tokens, hidden_size] residual stream, bf16 (float32 when hidden_is_fp32 != 0);
 *     delta: NULL or bf16 [tokens, hidden_size] added to it first (the last layer's MLP output,
 *             [tf]:781; rounded to bf16 when the stream is bf16), so only the slot rows of the
 *             last residual add are ever formed;
 *     slots (absolute token index), nopts: int32 [num_slots]; letters: [num_letters, hidden_size];
 *     probs, logits: float32 [num_slots, num_letters] (options >= nopts get p = 0, logit -inf).
 */
int fdk_slot_readout(const void* hidden, int hidden_is_fp32, const void* delta, int64_t hidden_size,
                     const int32_t* slots, const int32_t* nopts, int64_t num_slots,
                     const void* final_norm_w, int weight_is_fp32, const void* letters,
                     int64_t num_letters, float eps, float temperature, float* probs, float* logits,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FASTDECISIONS_B200_FDK_H_ */
