/*
 * dspark_b200.h - C ABI of the B200 (sm_100a) DSpark draft/verify attention library.
 *
 * All tensors are device pointers on the calling thread's current CUDA device;
 * every launch goes to `stream`. Shapes follow the Qwen3-0.6B attention of the
 * reference: 16 query heads, 8 KV heads, head dim 128, packed "THD" rows:
 *   queries  [total_q, 16, 128]      keys/values  [rows, 8, 128]
 * Query head h reads KV head h / 2 (GQA). `cu_q`/`cu_k` are int32 cumulative
 * row offsets with num_requests + 1 entries, as in the reference's PackedLayout.
 *
 * Return value: DSPARK_OK or an error status; nothing is launched when an
 * argument check fails. Values inside device arrays are not read on the host;
 * kernels that meet an out-of-range index skip it and set a bit in the device
 * status word (dspark_read_device_status). No entry point allocates memory;
 * bf16 attention needs a caller-owned workspace of
 * dspark_attention_workspace_size() bytes, which calls on one stream may share.
 */
#ifndef DSPARK_B200_H_
#define DSPARK_B200_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSPARK_ABI_VERSION 18

#define DSPARK_OK 0
#define DSPARK_ERR_INVALID_ARGUMENT 1
#define DSPARK_ERR_UNSUPPORTED 2
#define DSPARK_ERR_CUDA 3

#define DSPARK_DTYPE_BF16 0
#define DSPARK_DTYPE_F32 1

/* Device status bits (set by kernels, read with dspark_read_device_status). */
#define DSPARK_DEVICE_WAIT_TIMEOUT 1u
#define DSPARK_DEVICE_BAD_SCHEDULE 2u
#define DSPARK_DEVICE_BAD_ARGUMENT 4u

int dspark_abi_version(void);
const char* dspark_status_string(int status);

/* Number of kernels this library has launched since it was loaded (all devices
 * and streams); lets a caller count the library's launches in a timed region. */
unsigned long long dspark_launch_count(void);

/* Bytes of workspace the bf16 attention entry points need on `device`
 * (fp32 partials of items split between CTAs plus one merge record per CTA and
 * KV head; scales with the SM count, ~19 MB on a B200). Its contents never need
 * clearing: every launch rewrites the records it reads. Each bf16 attention
 * call launches the attention kernel and then the merge of its split items on
 * the same stream. */
int dspark_attention_workspace_size(int device, size_t* bytes);

/* Copies the device status word of the current device (synchronising), and
 * clears it when `clear` is non-zero. */
int dspark_read_device_status(unsigned int* status, int clear);

/* Enqueues on `stream` a copy of the current device's status word into `dst`
 * (pinned host or device memory), without synchronising: a decode loop that runs
 * ahead of the host reads it with the round's results. No reference counterpart
 * (the reference's kernels raise on the host instead). */
int dspark_copy_device_status(unsigned int* dst, cudaStream_t stream);

/*
 * Non-causal packed varlen attention: every query row of request i sees all
 * keys rows [cu_k[i], cu_k[i+1]).
 * Replaces PinnedRocmDraftKernel.__call__ (dspark_qwen/packed_draft.py:23-32),
 * i.e. aten::_flash_attention_forward(q, k, v, cu_q, cu_k, max_q, max_k, 0.0,
 * is_causal=False, ...); CPU oracle test_only_noncausal_varlen (packed_draft.py:35-47).
 * dtype DSPARK_DTYPE_BF16 (tensor cores) or DSPARK_DTYPE_F32 (exact CUDA-core path).
 * key_rows = rows of k/v (>= cu_k[num_requests]); max_q/max_k as in the reference call.
 */
int dspark_draft_attn(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                      int num_requests, int total_q, long long key_rows, int max_q, int max_k, float scale,
                      int dtype, void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Bottom-right causal packed varlen attention: query r of a request with q
 * queries and k keys sees key j iff j <= k - q + r. Rows of k/v after
 * cu_k[num_requests] (a capacity tail, key_rows beyond it) are never read.
 * Replaces PinnedRocmVarlenKernel.__call__ (dspark_qwen/rocm_varlen.py:108-117)
 * and the capacity-tail call PersistentQwenTarget._native_attention
 * (dspark_qwen/persistent_qwen_target.py:223-234); CPU oracles
 * test_only_dense_varlen (varlen_target.py:98-112) and test_only_persistent_sdpa
 * (persistent_qwen_target.py:30-42).
 */
int dspark_varlen_attn(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                       int num_requests, int total_q, long long key_rows, int max_q, int max_k, float scale,
                       int dtype, void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Two-source attention without a gather copy: keys of request i are rows
 * [a_off + a_start[i], + a_len[i]) of (ka, va) followed by rows
 * [b_off + b_start[i], + b_len[i]) of (kb, vb). kb == NULL drops the second
 * source; b_start == NULL means b_off + cu_q[i] and b_len == NULL means the
 * request's query count (the verify-scratch convention). causal selects the
 * bottom-right mask over the concatenated keys.
 * Replaces the concat + index_select + kernel call of PackedDraft.backbone
 * (dspark_qwen/packed_draft.py:215-236), the resident+scratch gather of
 * PersistentTargetKV.prepare_attention (persistent_target_kv.py:441-460) feeding
 * _native_attention, and the training-layout block-mask SDPA of
 * DraftAttention.forward with block_mask (dspark_qwen/model.py:12-19,47-61)
 * when each block is one request (context rows [0, anchor) + its 7 block rows).
 */
int dspark_segment_attn(const void* q, const void* ka, const void* va, long long rows_a, const void* kb,
                        const void* vb, long long rows_b, const int32_t* cu_q, const int32_t* a_start,
                        const int32_t* a_len, const int32_t* b_start, const int32_t* b_len, int a_off, int b_off,
                        int num_requests, int total_q, int max_q, int causal, float scale, int dtype, void* out,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * cos/sin table of a verify transaction, shared by every layer: new row r of
 * request i (row cu_q[i] + r) is at position p = ctx_len[i] + r, and
 * table[row * 64 + f] = rope_cache[p * 64 + f] for the 64 frequencies f.
 * rope_cache: [cache_rows, 64] uint32 (bf16 cos in the low half, bf16 sin in the
 * high half, of float32(p) * inv_freq[f]) that the caller evaluates once per model,
 * on the host, with the float32 ops of its rotary module; the Python layer builds
 * it with torch's CPU cos/sin, which is what transformers' Qwen3RotaryEmbedding
 * runs on the reference's CPU path, so the kernels' RoPE is bit-identical to it.
 * table: [total_q, 64] uint32; both 16-byte aligned. A position >= cache_rows
 * yields a zero row and sets DSPARK_DEVICE_BAD_ARGUMENT. Replaces the per-forward
 * Qwen3RotaryEmbedding.forward of transformers (modeling_qwen3.py:137-148) that
 * the reference's verify runs once per model call (persistent_qwen_target.py:408-410).
 */
int dspark_rope_table(const void* rope_cache, int cache_rows, const int32_t* cu_q, const int32_t* ctx_len,
                      int num_requests, int total_q, void* table, cudaStream_t stream);

/*
 * Verify layer for a persistent KV store (bf16):
 *  1. Qwen3 q_norm/k_norm (RMSNorm over the head dim, eps) and rotate-half RoPE
 *     (cos/sin from dspark_rope_table) of the new tokens' raw projections, at
 *     position ctx_len[i] + r for new row r of request i;
 *  2. KV append: roped k and raw v into scratch rows layer*scratch_rows + cu_q[i] + r;
 *  3. bottom-right causal attention over the resident prefix rows
 *     layer*rows_per_layer + slot_row[i] + [0, ctx_len[i]) followed by the
 *     request's new rows, read in place (no workspace gather);
 *  4. the merge of requests split between CTAs.
 * `path` DSPARK_VERIFY_FUSED does 1-3 in one attention kernel (q normalised in
 * registers, new k in shared memory after its TMA load); DSPARK_VERIFY_PREP runs
 * 1-2 as a small kernel once per new row (q written to `out`, which the
 * attention kernel then reads in place) and the attention as its programmatic
 * dependent, which pays off for small launches where every CTA would repeat
 * the q prologue; DSPARK_VERIFY_AUTO takes PREP below 512 new rows or when a
 * request has more than 16 (prefill chunks). Resident
 * K/V: [num_layers * rows_per_layer, 8, 128]; scratch K/V:
 * [num_layers * scratch_rows, 8, 128]; k_raw/v_raw: [total_q, 8, 128].
 * Replaces, per decoder layer, transformers Qwen3Attention.forward's
 * q_norm/k_norm/apply_rotary_pos_emb (modeling_qwen3.py:263-268) plus
 * _VerificationCache.update (dspark_qwen/persistent_qwen_target.py:73-83:
 * PersistentTargetKV.stage_layer + prepare_attention, persistent_target_kv.py:427-460)
 * plus persistent_attention_forward -> _native_attention (persistent_qwen_target.py:45-60,223-234).
 */
#define DSPARK_VERIFY_AUTO (-1)
#define DSPARK_VERIFY_FUSED 0
#define DSPARK_VERIFY_PREP 1
int dspark_verify_fused(const void* q_raw, const void* k_raw, const void* v_raw, const void* q_norm_weight,
                        const void* k_norm_weight, const void* rope_table, float eps, const int32_t* cu_q,
                        const int32_t* slot_row, const int32_t* ctx_len, int num_requests, int total_q, int max_q,
                        void* resident_k, void* resident_v, long long rows_per_layer, void* scratch_k,
                        void* scratch_v, int scratch_rows, int num_layers, int layer, float scale, int path,
                        void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * dspark_verify_fused with row strides (elements) for the q/k/v projections, e.g.
 * column blocks of one merged [n, (16 + 8 + 8) * 128] q|k|v GEMM output, so a host
 * runs one projection GEMM per layer instead of three. Strides must be multiples
 * of 8 and at least the packed row (16 * 128, 8 * 128, 8 * 128). Packed strides
 * behave exactly as dspark_verify_fused; other strides take the prep path (its
 * kernel reads the strided rows and writes packed q and scratch K/V), and
 * path == DSPARK_VERIFY_FUSED with them is refused.
 */
int dspark_verify_strided(const void* q_raw, long long ld_q, const void* k_raw, long long ld_k, const void* v_raw,
                          long long ld_v, const void* q_norm_weight, const void* k_norm_weight,
                          const void* rope_table, float eps, const int32_t* cu_q, const int32_t* slot_row,
                          const int32_t* ctx_len, int num_requests, int total_q, int max_q, void* resident_k,
                          void* resident_v, long long rows_per_layer, void* scratch_k, void* scratch_v,
                          int scratch_rows, int num_layers, int layer, float scale, int path, void* out,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Commit / rollback for all layers in one launch: for every request copy
 * scratch rows [cu_q[i], cu_q[i] + n_commit[i]) of each layer into resident rows
 * slot_row[i] + [ctx_len[i], ctx_len[i] + n_commit[i]). Rows past n_commit
 * (the rejected drafts) are not copied, which is the rollback. Requires
 * 0 <= n_commit[i] <= q_i and ctx_len[i] + n_commit[i] <= slot_cap[i]. dtype: the
 * element type of the K/V rows (DSPARK_DTYPE_BF16 or DSPARK_DTYPE_F32).
 * Replaces PersistentTargetKV.commit (dspark_qwen/persistent_target_kv.py:463-491);
 * abort (493-499) needs no device work.
 */
int dspark_commit_kv(void* resident_k, void* resident_v, const void* scratch_k, const void* scratch_v,
                     const int32_t* cu_q, const int32_t* slot_row, const int32_t* ctx_len, const int32_t* slot_cap,
                     const int32_t* n_commit, int num_requests, int num_layers, long long rows_per_layer,
                     int scratch_rows, int dtype, cudaStream_t stream);

/*
 * On-device greedy acceptance of a verify round (the rule of
 * dspark_qwen/cached_decode.py:84-98; the reference applies it on the host).
 *
 * dspark_row_argmax: pred[r] = index of the maximum of logits row r (rows x vocab,
 * row stride ld elements, bf16 or fp32); ties give the lowest index and NaN is
 * larger than any number (torch.argmax).
 *
 * dspark_greedy_accept: request i verified the chunk tokens[cu_q[i]..cu_q[i+1]-1]
 * (anchor, then its proposals) and pred holds the target's prediction after each
 * of those rows. Proposals are accepted while they equal the prediction before
 * them (stopping after an accepted EOS); the first mismatch commits the target's
 * token instead and a full accept commits the bonus prediction. Committed tokens
 * are cut after their first EOS and to budget[i] (if budget is not NULL). Outputs:
 * accepted[i] proposals, n_commit[i] committed tokens (= verified rows to keep,
 * the n_commit input of dspark_commit_kv) and emitted[cu_q[i] + k] the committed
 * tokens (-1 after them). All pointers are device memory; int64 tokens.
 */
int dspark_row_argmax(const void* logits, long long ld, int rows, int vocab, int dtype, int32_t* pred,
                      cudaStream_t stream);
int dspark_greedy_accept(const int32_t* pred, const long long* tokens, const int32_t* cu_q, int num_requests,
                         int total_rows, const long long* eos, int n_eos, const int32_t* budget, int32_t* accepted,
                         int32_t* n_commit, long long* emitted, cudaStream_t stream);

/*
 * Qwen3RMSNorm.forward of bf16 rows in one launch (the target's input_layernorm,
 * post_attention_layernorm and final norm; transformers 5.5
 * models/qwen3/modeling_qwen3.py:62-66, run by the reference's target forward in
 * dspark_qwen/persistent_qwen_target.py and its draft blocks in
 * dspark_qwen/model.py:67-86). For each of rows rows of hidden elements
 * (row strides ld_x / ld_out elements):
 *   r = rsqrtf(sum(x*x) * fl(1/hidden) + eps),  out = bf16(w * bf16(x * r))
 * rounded step by step as the torch sequence is; only the order of the float sum
 * differs. Requires hidden % 8 == 0, strides that are multiples of 8 and 16-byte
 * aligned x, weight and out; rows == 0 launches nothing (pointers may then be
 * NULL). All device memory.
 */
int dspark_rms_norm(const void* x, long long ld_x, const void* weight, float eps, int rows, int hidden, void* out,
                    long long ld_out, cudaStream_t stream);

/*
 * Residual add + Qwen3RMSNorm in one launch (bf16): sum_out = bf16(x + delta),
 * torch's bf16 add of a decoder layer's residual and sublayer output, and out =
 * dspark_rms_norm(sum_out). Same rules as dspark_rms_norm for every pointer and
 * stride; x and delta must not overlap out or sum_out, nor out sum_out: such a call
 * (an in-place residual update, say) is refused with DSPARK_ERR_INVALID_ARGUMENT.
 */
int dspark_add_rms_norm(const void* x, long long ld_x, const void* delta, long long ld_d, const void* weight,
                        float eps, int rows, int hidden, void* out, long long ld_out, void* sum_out,
                        long long ld_sum, cudaStream_t stream);

/*
 * The draft block's q/k head norms and rotate-half RoPE in one launch (bf16,
 * head_dim 128; project_q / project_kv of dspark_qwen/model.py:41-45 with rotate,
 * model.py:22-24). Row i of q (row stride ld_q elements) holds q_heads heads, of k
 * (ld_k) kv_heads heads; cos_table / sin_table are the rotary module's bf16 rows
 * (stride ld_cs). Per head: y = Qwen3RMSNorm(x) as in dspark_rms_norm, then
 * out[d] = bf16(bf16(y[d] cos[d]) + bf16(rot[d] sin[d])) with rot = (-y[64:], y[:64]),
 * rounded where torch's bf16 ops round. Outputs packed [rows, heads, 128]. Strides
 * multiples of 4, 8-byte aligned pointers; rows == 0 launches nothing. Device memory.
 */
int dspark_qk_norm_rope(const void* q, long long ld_q, const void* k, long long ld_k, const void* q_norm_weight,
                        const void* k_norm_weight, float q_eps, float k_eps, const void* cos_table,
                        const void* sin_table, long long ld_cs, int rows, int q_heads, int kv_heads, void* q_out,
                        void* k_out, cudaStream_t stream);

/*
 * Gated activation of a Qwen3MLP from one merged [gate; up] projection (bf16):
 * row i of gate_up (stride ld elements) holds inter gate then inter up values;
 * out[i, c] = bf16(bf16(silu(g)) * u) with silu(g) = g / (1 + expf(-g)) in float,
 * as torch's silu and bf16 product round. Replaces act_fn(gate_proj(x)) *
 * up_proj(x) of transformers' Qwen3MLP.forward (two GEMMs and two elementwise
 * kernels) after a single GEMM. inter % 8 == 0, strides multiples of 8, 16-byte
 * aligned pointers; rows == 0 launches nothing. Device memory.
 */
int dspark_silu_mul(const void* gate_up, long long ld, int rows, int inter, void* out, long long ld_out,
                    cudaStream_t stream);

/*
 * One step of the draft's greedy Markov proposal (DSparkDraft._sample_greedy,
 * dspark_qwen/model.py:210-221), bf16, for up to 128 requests:
 *   emb = emb_table[prev[r * prev_stride]]                        (rank wide)
 *   conf[r * tok_stride + k] = sigmoid(hidden_row . conf_w[:H] + emb . conf_w[H:] + conf_b)
 *   tokens[r * tok_stride + k] = argmax_v(base_row[v] + emb . proj_weight[v])
 * where base_row / hidden_row are rows r * base_stride_r + k of base [*, vocab]
 * (the LM head logits of the block rows) and hidden [*, hidden_dim], with the
 * reference's bf16 rounding (projection output, then the sum) and ties to the
 * lowest index. proj_weight / emb_table are [vocab, rank] (vocab a multiple of 8,
 * rank a multiple of 64 up to 256). The [R, vocab] logits are never written:
 * a tcgen05 GEMM keeps each tile in TMEM and the argmax is folded in. scratch
 * (dspark_markov_scratch_bytes(), 16-byte aligned device memory) must be zero
 * before the first call and is kept usable by every call (one scratch per
 * stream). Run the block's steps k = 0 .. S-1 in order, passing prev = the
 * anchors for k = 0 and prev = tokens + (k - 1) (stride tok_stride) afterwards.
 *
 * dspark_markov_block runs all block_size (<= 64) steps of a block in one
 * cooperative launch (the same results as dspark_markov_step for k = 0 ..
 * block_size-1 with base_stride_r = tok_stride = block_size and prev = anchors
 * [num_requests]): the projection weight streams on across steps and the CTAs
 * meet at a bounded grid barrier between steps. If the cooperative launch is
 * refused (not every CTA could be resident), it launches the steps one by one.
 * A call whose barrier wait gives up (DSPARK_DEVICE_WAIT_TIMEOUT in the device
 * status) returns unusable tokens but leaves the scratch zero again: its last CTA
 * to finish resets it, so the next call on the stream is correct.
 */
size_t dspark_markov_scratch_bytes(void);

/*
 * Sets the time limit (nanoseconds of the GPU's global timer, on the current
 * device) of the grid barrier in dspark_markov_block; the default is two
 * seconds, like every other bounded wait of the library. A diagnostic for
 * failure handling: a test lowers it to make the barrier give up, checks the
 * status word and the next call, and puts it back. No reference counterpart.
 */
int dspark_set_grid_barrier_timeout(unsigned long long ns);
int dspark_markov_step(const void* proj_weight, const void* emb_table, int vocab, int rank, const void* base,
                       long long base_stride_r, int k, const long long* prev, long long prev_stride,
                       const void* hidden, int hidden_dim, const void* conf_w, float conf_b, long long* tokens,
                       float* conf, long long tok_stride, int num_requests, void* scratch, cudaStream_t stream);
int dspark_markov_block(const void* proj_weight, const void* emb_table, int vocab, int rank, const void* base,
                        int block_size, const long long* anchors, const void* hidden, int hidden_dim,
                        const void* conf_w, float conf_b, long long* tokens, float* conf, int num_requests,
                        void* scratch, cudaStream_t stream);

/*
 * Fused draft-context append (bf16, tcgen05 tensor cores): for every draft layer
 * l < num_layers, k = RoPE(k_norm_l(context @ k_proj_l^T)) and
 * v = context @ v_proj_l^T of each input row, written into the layer's K/V pool.
 * context: [rows, hidden] (the output of the draft's fc + context_norm; hidden a
 * multiple of 64); kv_weight: [num_layers * 2048, hidden], layer l's k_proj
 * weight rows then its v_proj weight rows; k_norm_weight: [num_layers, 128];
 * rope_table: [rows, 64] from dspark_rope_table over the same cu_rows / ctx_len.
 * Input row g of request i (cu_rows[i] <= g < cu_rows[i + 1], j = g - cu_rows[i])
 * is at position ctx_len[i] + j and lands in pool row slot_row[i] + ctx_len[i] + j
 * when j < count[i], else in trash_row (so whole verified chunks can be appended
 * with fixed shapes and only the committed rows become visible). pool_k / pool_v:
 * host arrays of num_layers (<= 8) device pointers, each [pool_rows, 8, 128];
 * destination rows outside [0, pool_rows) are skipped and flagged in the device
 * status. context, kv_weight, k_norm_weight, rope_table and every pool pointer
 * 16-byte aligned (DSPARK_ERR_INVALID_ARGUMENT otherwise). Arithmetic follows the
 * reference's bf16 ops (projection output, RMSNorm, weight product, each RoPE
 * product and the sum rounded to bf16).
 * Replaces PackedDraft.append_committed's per-layer project_kv and cache
 * concatenation (dspark_qwen/packed_draft.py:146-158; model.py:41-45).
 */
int dspark_draft_append(const void* context, int rows, int hidden, const void* kv_weight, int num_layers,
                        const void* k_norm_weight, const void* rope_table, float eps, const int32_t* cu_rows,
                        const int32_t* slot_row, const int32_t* ctx_len, const int32_t* count, int num_requests,
                        void* const* pool_k, void* const* pool_v, long long pool_rows, long long trash_row,
                        cudaStream_t stream);

/*
 * Stochastic acceptance of a verify round under the reference's float64 law
 * (dspark_qwen/tensor_sampling.py:38-162): for request i with n_i = cu_n[i+1] - cu_n[i]
 * proposals tokens[cu_n[i] ..] drawn from the draft laws q[cu_n[i] ..] ([draft_rows,
 * vocab] float64), the target laws are softmax(logits / temperature) in float64,
 * normalised once more, of target rows cu_n[i] + i .. + n_i (n_i + 1 rows of `logits`,
 * bf16 or f32, row stride ld). Proposal j is accepted while u < min(p[t] / q[t], 1); the
 * first rejection samples the residual law relu(p - q) / mass, a full accept samples the
 * last target row (strict CDF rule, last positive index past the end); an accepted EOS
 * stops the round, and so does reaching budget[i] tokens. Uniforms are consumed from
 * uniforms[i * u_stride ..] in the reference's draw order (u_stride >= n_i + 1).
 * Outputs: emitted[i * u_stride ..] (committed tokens, -1 after) and result[i * 8 ..] =
 * {count, accepted, rejected index or -1, extra (0 none, 1 residual, 2 bonus),
 *  reason (0 round complete, 1 EOS, 2 budget), uniforms used, status, 0}; status 0 or a
 * refusal of the reference's checks (1 non-finite logits, 2 draft row not a law, 3 token
 * out of range, 4 proposal with zero draft mass, 5 zero residual mass, 6 uniform outside
 * [0, 1), 7 inconsistent offsets), in which case count is 0. scratch: device memory of
 * dspark_stochastic_scratch_bytes(target_rows + draft_rows) bytes (the row
 * statistics and a 512 KB table of x / T for every bf16 bit pattern, so the
 * float64 passes read x / T instead of dividing). Three launches for bf16
 * logits (the table first), two for f32.
 */
size_t dspark_stochastic_scratch_bytes(int rows);

/*
 * Stochastic draft proposal of one Markov position for `rows` requests
 * (DSparkDraft._sample_stochastic, dspark_qwen/model.py:193-208, batched over
 * requests as packed_sampling.py:73-94 does; bf16 logits). Launch row r reads
 * request row i = row_index[r] (row_index NULL: i = r): its LM-head row at
 * base + i * ld_base and its Markov projection row at proj + r * ld_proj (bf16
 * elements); x = bf16(base + proj) as torch adds them. It writes the float64 law
 * q = softmax(x / T) normalised once more (logits_to_probabilities,
 * tensor_sampling.py:38-51) to law + i * ld_law, draws one token with uniforms[r]
 * by the strict CDF rule, the last positive index past the end
 * (sample_categorical, tensor_sampling.py:77-84), into tokens[r], and sets
 * status[r] to 0, or 1 when x / T is not finite. Scratch of
 * dspark_propose_scratch_bytes() bytes (the x / T table of the 65536 bf16 bit
 * patterns, rebuilt per call), 16-byte aligned; law 8-byte aligned. rows == 0
 * launches nothing. Device memory.
 */
size_t dspark_propose_scratch_bytes(void);
int dspark_stochastic_propose(const void* base, long long ld_base, const int32_t* row_index, const void* proj,
                              long long ld_proj, int vocab, double temperature, const double* uniforms, int rows,
                              double* law, long long ld_law, long long* tokens, int32_t* status, void* scratch,
                              size_t scratch_bytes, cudaStream_t stream);
int dspark_stochastic_accept(const void* logits, long long ld, int dtype, int vocab, double temperature,
                             int target_rows, const double* q, int draft_rows, const long long* tokens,
                             const int32_t* cu_n, int num_requests, const double* uniforms, int u_stride,
                             const long long* eos, int n_eos, const int32_t* budget, long long* emitted,
                             int32_t* result, void* scratch, size_t scratch_bytes, cudaStream_t stream);

/*
 * Training-layout block-draft attention (bf16, tcgen05 tensor cores).
 * Replaces DraftAttention.forward's masked SDPA with block_mask
 * (dspark_qwen/model.py:12-19,47-61) for several sequences packed back to back.
 * Sequence s has ctx_len[s] context rows and num_blocks[s] anchors (its slice
 * of `anchors`, in order); its queries are num_blocks[s]*block_size rows, its
 * keys are [ctx_len[s] context rows ; the same block rows]. Block b's rows see
 * context rows j < anchors[b] (anchors are clamped to [0, ctx_len[s]], which is
 * what the mask does) and all rows of block b; sequences never see each other.
 *
 * dspark_train_plan runs on the host only (all pointers are HOST memory): it
 * splits the queries into 64-row tiles per KV head and assigns them to at most
 * grid_limit persistent CTAs (largest first onto the least-loaded CTA). Call it
 * with plan == NULL to get the plan size in int32 words in *plan_words; the
 * plan is then copied to the device once and reused by every call with the
 * same layout. Returns DSPARK_ERR_UNSUPPORTED if the packed sizes reach 2^31.
 * block_size must be in [6, 32].
 *
 * dspark_train_attn launches plan[2] CTAs (`grid` must equal it) on q
 * [total_q, 16, 128], k/v [total_k, 8, 128] and writes out [total_q, 16, 128]
 * (all bf16, 16-byte aligned, device memory; plan 16-byte aligned device
 * memory). A plan built for other sizes sets DSPARK_DEVICE_BAD_ARGUMENT and
 * computes nothing.
 */
int dspark_train_plan(int num_seqs, const int32_t* ctx_len, const int32_t* num_blocks, const int32_t* anchors,
                      int block_size, int grid_limit, int32_t* plan, long long plan_capacity, long long* plan_words);
int dspark_train_attn(const void* q, const void* k, const void* v, int total_q, long long total_k,
                      const int32_t* plan, int grid, float scale, void* out, cudaStream_t stream);

/*
 * Allocation-free variant of dspark_varlen_attn (bf16 only). No counterpart in
 * the reference: it exists for callers that cannot allocate device memory for a
 * workspace - an FFI host (Go, Java) without access to the allocator that owns
 * the GPU, or a server that has reserved nearly all HBM for its KV-cache pool,
 * where an extra cudaMalloc would fail and a cudaMalloc/cudaFree would stall the
 * device mid-step. The split-item scratch is a static device array of
 * dspark_varlen_attn_noalloc_scratch_bytes() bytes (18.8 MiB: partials and
 * merge records of at most 148 CTAs) that every GPU loading the library holds until exit; the
 * requirement does not grow with the inputs, and the call returns
 * DSPARK_ERR_UNSUPPORTED if a launch would ever need more. The first call on a
 * device looks up that device's address of the array (make it before any
 * stream capture). All calls share the array and it keeps the last call's
 * contents (nothing in it needs to start at zero); calls that overlap on the
 * GPU, e.g. on two streams, race on it. Allocates nothing.
 */
size_t dspark_varlen_attn_noalloc_scratch_bytes(void);
int dspark_varlen_attn_noalloc(const void* q, const void* k, const void* v, const int32_t* cu_q,
                               const int32_t* cu_k, int num_requests, int total_q, long long key_rows, int max_q,
                               int max_k, float scale, void* out, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* DSPARK_B200_H_ */
