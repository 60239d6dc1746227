/*
 * std_b200.h -- C ABI of the B200 (sm_100a) STD sparse-to-dense decode path.
 *
 * Conventions for every entry point:
 *   - all tensor pointers are caller-owned DEVICE pointers (bf16 = 16-bit
 *     bfloat16 bit patterns, contiguous, 16-byte aligned unless stated);
 *   - `stream` is a cudaStream_t (passed as void*); work is enqueued only,
 *     nothing synchronises, and every launch is CUDA-graph capturable;
 *   - return value: 0 ok; 1 bad shape/argument; 2 capacity exceeded;
 *     3 unsupported device / driver entry point missing; 4 CUDA launch error;
 *     5 workspace missing or too small.  No exceptions cross the ABI;
 *   - lengths are device-resident int32 arrays (one entry per request), so a
 *     decode round never reads them on the host;
 *   - kernels never allocate; scratch memory is a caller-provided workspace
 *     whose size is given by the matching *_workspace_bytes() function.  It
 *     needs no initialisation and must not be shared by launches that can
 *     run concurrently;
 *   - device-side faults are never raised: a wait that exceeds its ~1 s limit
 *     or an out-of-range index is recorded in a device error word that
 *     std_get_device_error() reads and clears.
 *
 * KV cache layout (both caches): [layers, 2 (K,V), B, Hkv, cap, D] bf16, so
 * the K (or V) cache of one layer is a contiguous [B, Hkv, cap, D] block.
 * Reference counterparts are cited as path:line of mcy1123/STD.
 */
#ifndef STD_B200_H
#define STD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- library ---------------------------------------------------------- */

/* Library version (major*10000 + minor*100 + patch). */
int std_version(void);

/* Reads and clears the device error word of the current device
 * (0 none, 1 wait timeout, 2 index out of bounds skipped, 3 length > capacity). */
int std_get_device_error(int* code_out);

/* 1 when the current device is sm_100 (B200), else 0. */
int std_device_supported(void);

/* ---- (b) sparse draft attention --------------------------------------- */

/* Replaces: std_qwen25vl.py:406-417 (F.scaled_dot_product_attention(q, k, v,
 * enable_gqa=True), q_len = 1) and triton_attention.py:83-112
 * (fused_gqa_attention(q, k, v)).
 * q [B, Hq, D]; k_cache / v_cache: one layer's [B, Hkv, cap, D]; request b
 * attends to keys 0 .. lens[b]+len_offset-1 (no mask); out [B, Hq, D] bf16;
 * lse [B, Hq] fp32 natural-log (optional, may be NULL).  Hq = 7*Hkv, D = 128. */
size_t std_draft_attn_workspace_bytes(int B, int Hq, int Hkv, int D, int cap);
/* flags: 0, or STD_DRAFT_AFTER_APPEND when the launch just before this one on
 * `stream` writes nothing this call reads except q and, per request, the K/V
 * row at position lens[b]+len_offset-1 (a decode step's RoPE + KV append).
 * The kernel then reads the lengths and the older K/V rows while that launch
 * may still be running (programmatic dependent launch). */
#define STD_DRAFT_AFTER_APPEND 1
int std_draft_attn(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens, int len_offset,
                   int B, int Hq, int Hkv, int D, int cap, void* out, float* lse, void* workspace,
                   size_t workspace_bytes, int flags, void* stream);

/* Index-based sparse cache (the reference's unused gather variant,
 * std_qwen25vl.py:323-351, made the draft path): request b, KV head h attends
 * to dense_k/v rows idx[b][h][0 .. n_idx) (ascending prompt positions of this
 * layer's selection, read in place from the dense cache [B, Hkv, cap_dense, D])
 * followed by rows 0 .. L-n_idx-1 of the tail [B, Hkv, tail_cap, D] that holds
 * the generated tokens' draft-path K/V; L = lens[b]+len_offset.  Same result,
 * byte for byte, as std_draft_attn over the compacted copy of those rows. */
int std_draft_attn_indexed(const void* q, const void* dense_k, const void* dense_v, int cap_dense,
                           const int32_t* idx, int n_idx, const void* tail_k, const void* tail_v, int tail_cap,
                           const int32_t* lens, int len_offset, int B, int Hq, int Hkv, int D, void* out, float* lse,
                           void* stream);

/* ---- (c) parallel dense verify attention (also AR dense decode, nq = 1) -- */

/* Replaces: modeling_qwen2_5_vl.py:1096-1133 (repeat_kv + F.sdpa with the
 * causal mask of :65-101) in the verify forward std_qwen25vl.py:797-803 and in
 * the AR loop std_qwen25vl.py:584-590.
 * q [B, nq, Hq, D] (token-major); L = lens[b]+len_offset keys (the nq new
 * tokens' keys already appended); causal=1: token t sees keys 0 .. L-nq+t;
 * causal=0: every token sees all L keys (a sequence shard that holds only
 * past keys).  out [B, nq, Hq, D] bf16; lse [B, nq, Hq] fp32 (optional).
 * 1 <= nq <= 18, Hq = 7*Hkv, D = 128.  Rows are bit-identical for any nq. */
size_t std_verify_attn_workspace_bytes(int B, int Hkv, int cap);
int std_verify_attn(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens, int len_offset,
                    int nq, int causal, int B, int Hq, int Hkv, int D, int cap, void* out, float* lse,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Same computation as std_verify_attn, for callers that cannot allocate device
 * memory (a serving process that keeps the whole GPU in its own pool and does
 * not let plugins allocate; an FFI caller with no device allocator; a loop
 * that cannot afford an allocation's device synchronisation).  It has no
 * counterpart in the reference.  Its scratch is a fixed array of
 * STD_VERIFY_NOALLOC_SCRATCH_BYTES inside this library, held on every GPU
 * that loads the library until the process exits; the call allocates
 * nothing.  Shapes whose scratch (std_verify_attn_workspace_bytes) exceeds
 * that size are rejected with status 2.  The first call on a device looks up
 * the array's device address with that device current; make that first call
 * before any stream capture.  All calls share the one array: calls that can
 * overlap on the GPU (other streams, other host threads on the same device)
 * race and must be serialised by the caller.  Nothing in the array needs to
 * start at zero. */
#define STD_VERIFY_NOALLOC_SCRATCH_BYTES (32u << 20)
int std_verify_attn_noalloc(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                            int len_offset, int nq, int causal, int B, int Hq, int Hkv, int D, int cap, void* out,
                            float* lse, void* stream);

/* std_verify_attn with an fp32 output (out_f32 [B, nq, Hq, D]) and a
 * required natural-log LSE: the partial of one key range for a
 * sequence-sharded verify, merged with std_merge_partials_f32 (no reference
 * counterpart). */
int std_verify_attn_partial(const void* q, const void* k_cache, const void* v_cache, const int32_t* lens,
                            int len_offset, int nq, int causal, int B, int Hq, int Hkv, int D, int cap, float* out_f32,
                            float* lse, void* workspace, size_t workspace_bytes, void* stream);
/* Exact (O, LSE) merge of fp32 partials packed one buffer per part: part i
 * is [rows * D O | rows LSE] at parts + i * part_stride floats; out [rows, D]
 * bf16, lse_out [rows] (optional).  The merge step of sequence-sharded verify
 * after one all-gather of the packed partials. */
int std_merge_partials_f32(const float* parts, long long part_stride, int n_parts, int rows, int D, void* out,
                           float* lse_out, void* stream);
/* Exact (O, LSE) merge of attention partials computed over disjoint key
 * ranges (sequence shards).  Replaces nothing in the reference (it has no
 * sequence parallelism); it is the exchange step of sharded verify.
 * o_parts [n_parts, rows, D] bf16, lse_parts [n_parts, rows] fp32 ->
 * out [rows, D] bf16, lse_out [rows] (optional). */
int std_merge_partials(const void* o_parts, const float* lse_parts, int n_parts, int rows, int D, void* out,
                       float* lse_out, void* stream);

/* ---- (a) prefill-time selection ---------------------------------------- */

/* Replaces: modeling_qwen2_5_vl.py:966-995 (custom fp16 attention weights for
 * output_attentions=True) + std_qwen25vl.py:204-218 (grouped fp32 sum).
 * q_text [T, Hq, D] bf16 (text rows, after RoPE); k_cache [Hkv, kstride, D]
 * bf16 (one request, one layer, rows 0..P-1); row t sits at absolute position
 * q_start+t and sees keys 0..q_start+t.  scores [Hkv, P] fp32.
 * write_probs=1 leaves the fp16 probabilities in the workspace as
 * [Hq, T, pstride] (pstride from std_select_probs_view) for the selection
 * branch's attention output. */
size_t std_select_workspace_bytes(int T, int Hq, int P);
int std_select_scores(const void* q_text, const void* k_cache, long long kstride, int T, int Hq, int Hkv, int D,
                      int P, int q_start, float scale, float* scores, int write_probs, void* workspace,
                      size_t workspace_bytes, void* stream);
int std_select_probs_view(int T, int Hq, int P, long long* pstride_out);

/* Replaces: std_qwen25vl.py:219-222 (index_select visual columns, torch.topk,
 * map to positions, sort).  For each of n_seg score rows (stride seg_stride):
 * the K largest scores among visual_pos[0..V-1] (ascending absolute
 * positions), ties to the lowest position, written ascending to out[n_seg, K]. */
int std_topk_select(const float* scores, long long seg_stride, int n_seg, const int32_t* visual_pos, int V, int K,
                    int32_t* out, void* stream);

/* Replaces: std_qwen25vl.py:265-298 (compact_sparse_prompt_cache) and
 * :301-320 (copy_prompt_cache).  For request b and every layer and KV head,
 * slot j of the sparse cache receives dense row idx[j] where
 * idx = sorted(non_visual U topk[layer, head]) (disjoint sets). */
int std_compact_gather(const void* dense_cache, void* sparse_cache, int layers, int B, int b, int Hkv, int D,
                       int cap_dense, int cap_sparse, const int32_t* non_visual, int NV, const int32_t* topk, int K,
                       void* stream);

/* ---- decoder pieces around the library GEMMs --------------------------- */

/* modeling_qwen2_5_vl.py:1336 (embed_tokens): out[b*n+j] = table[tok[b*tok_stride+tok_start+j]]. */
int std_embed(const void* table, int vocab, int H, const int32_t* tok, int tok_stride, int tok_start, int n, int B,
              void* out, void* stream);
/* modeling_qwen2_5_vl.py:183-197 (Qwen2RMSNorm).  H % 8 == 0, H/8 <= 512. */
int std_rmsnorm(const void* x, const void* w, float eps, int M, int H, void* out, void* stream);
/* modeling_qwen2_5_vl.py:1200-1221 + :183-197 (residual add, then the next
 * RMSNorm): x <- bf16(x + delta) in place, out = rmsnorm(x) * w. */
int std_add_rmsnorm(void* x, const void* delta, const void* w, float eps, int M, int H, void* out, void* stream);
/* modeling_qwen2_5_vl.py:690-732 (RoPE, 1-D positions) + kv_cache.py:54-69
 * (KVCache.cat): rotates q and k of qkv [B*n, (Hq+2Hkv)*D], writes q_out and
 * appends k, v at cache slot slot_base[b]+slot_off+j, position
 * pos_base[b]+pos_off+j, cos/sin tables [max_pos, D/2] bf16. */
int std_rope_append(const void* qkv, int B, int n, int Hq, int Hkv, int D, const int32_t* pos_base, int pos_off,
                    const int32_t* slot_base, int slot_off, const void* cos_t, const void* sin_t, int max_pos,
                    void* q_out, void* k_cache, void* v_cache, int cap, void* stream);
/* modeling_qwen2_5_vl.py:674-687 (Qwen2MLP act_fn(gate) * up): gu rows of 2I
 * columns, [gate | up] halves, or with interleaved != 0 64-feature
 * [gate | up] blocks (I % 64 == 0); out [M, I]. */
int std_silu_mul(const void* gu, int M, int I, int interleaved, void* out, void* stream);
/* residual add (modeling_qwen2_5_vl.py:1200-1221). */
int std_add(const void* a, const void* b, size_t n, void* out, void* stream);
/* std_qwen25vl.py:98-99, :806 (torch.argmax, first index on ties):
 * out[(row/n)*out_stride + out_start + row%n] = argmax(logits[row, :V]).  V % 8 == 0. */
int std_argmax_rows(const void* logits, int rows, int V, int n, int out_stride, int out_start, int32_t* out,
                    void* stream);

/* Decode-time linear layer: y[M, N] = x[M, K] . w[N, K]^T (+ bias[N]), bf16,
 * fp32 accumulation, tcgen05 weight streaming; replaces the cuBLAS GEMMs of
 * the decode forwards (modeling_qwen2_5_vl.py:778-781 q/k/v/o projections,
 * :674-687 Qwen2MLP, :1749 lm_head).  M <= 256, K % 64 == 0, N % 4 == 0.
 * A row's result does not depend on the other rows for a fixed M.  The
 * workspace holds split-K partials (0 bytes when the shape needs none). */
size_t std_gemm_workspace_bytes(int M, int N, int K);
int std_gemm_bf16(const void* x, const void* w, const void* bias, void* y, int M, int N, int K, void* workspace,
                  size_t workspace_bytes, void* stream);

/* GEMMs fused with the decode op that consumes them: the GEMM's bf16 result
 * goes through `workspace` (>= std_gemm_epilogue_workspace_bytes) straight
 * into the epilogue kernel, with the same arithmetic as the unfused pair.
 * N % 8 == 0. */
size_t std_gemm_epilogue_workspace_bytes(int M, int N, int K);
/* Replaces: the o_proj / down_proj output, the residual add and the next
 * RMSNorm of a decoder layer (modeling_qwen2_5_vl.py:1200-1221, Qwen2RMSNorm
 * :183-197):  resid <- bf16(resid + bf16(x . w^T + bias));
 * out = rmsnorm(resid) * norm_w.  norm_w == NULL: the residual add only.
 * Same result as std_gemm_bf16 followed by std_add_rmsnorm.  N/8 <= 512. */
int std_gemm_add_rmsnorm(const void* x, const void* w, const void* bias, void* resid, const void* norm_w, float eps,
                         void* out, int M, int N, int K, void* workspace, size_t workspace_bytes, void* stream);
/* Replaces: Qwen2MLP's act_fn(gate_proj(x)) * up_proj(x)
 * (modeling_qwen2_5_vl.py:674-687): act[M, I] from x [M, K] and the fused
 * gate/up weights w [2I, K] stored as 64-row [gate | up] blocks (a checkpoint
 * loader interleaves gate_proj and up_proj rows that way), without storing
 * the [M, 2I] intermediate.  Same result as std_gemm_bf16 followed by
 * std_silu_mul(interleaved = 1).  I % 64 == 0. */
int std_gemm_silu_mul(const void* x, const void* w, int M, int I, int K, void* act, void* workspace,
                      size_t workspace_bytes, void* stream);
/* Replaces: lm_head (modeling_qwen2_5_vl.py:1749) + the greedy argmax of the
 * decode loops (std_qwen25vl.py:98-99, :806): for the first rows_out rows of
 * x [M, K] . w [N, K]^T, out[(t/n)*out_stride + out_start + t%n] = first
 * column of the maximum bf16 logit, without storing the logits.  keys: M
 * uint64 scratch, all zero on entry (zero it once before the first call); the
 * call leaves it zero.  Same result as std_gemm_bf16 + std_argmax_rows.
 * margin_out (optional, fp32, indexed like out): the row's largest minus
 * second-largest logit (verification_policy.py:29-46; equal maxima give 0). */
int std_gemm_argmax(const void* x, const void* w, int M, int N, int K, int rows_out, int n, int out_stride,
                    int out_start, int32_t* out, float* margin_out, unsigned long long* keys, void* workspace,
                    size_t workspace_bytes, void* stream);
/* Replaces: q/k/v_proj of a decode step (modeling_qwen2_5_vl.py:1050-1052),
 * RoPE (:690-732) and KVCache.cat (kv_cache.py:54-69): qkv = x . w^T + bias
 * (w [(Hq+2Hkv)*D, K]) then, per token row, the std_rope_append step on it.
 * Same result as std_gemm_bf16 followed by std_rope_append. */
int std_gemm_rope_append(const void* x, const void* w, const void* bias, int K, int B, int n, int Hq, int Hkv, int D,
                         const int32_t* pos_base, int pos_off, const int32_t* slot_base, int slot_off,
                         const void* cos_t, const void* sin_t, int max_pos, void* q_out, void* k_cache,
                         void* v_cache, int cap, void* workspace, size_t workspace_bytes, void* stream);

/* ---- (e) sequence-sharded verify over peer memory (one node) ---------- */

/* No reference counterpart (the reference has no sequence parallelism): the
 * exchange of the sequence-sharded verify without collectives.  Buffers that
 * another rank maps come from std_device_alloc (zero-filled cudaMalloc, so
 * their base can be exported); std_ipc_handle writes the allocation's
 * std_ipc_handle_bytes()-byte handle, std_ipc_open maps a peer's handle
 * (peer access enabled lazily), std_ipc_close unmaps it.  Every rank must be
 * a process on its own GPU of the same node. */
size_t std_ipc_handle_bytes(void);
int std_device_alloc(size_t bytes, void** ptr_out);
int std_device_free(void* ptr);
int std_ipc_handle(const void* base, void* handle_out);
int std_ipc_open(const void* handle, void** ptr_out);
int std_ipc_close(void* ptr);
/* Copy `bytes` (multiple of 16, may be 0) from src to dst on this GPU, then
 * publish epoch e = ++*counter (a device int of this rank) to each of the
 * n_flags <= 8 device ints `flags` (typically peers' flags) with system-scope
 * release stores, after the copy. */
int std_p2p_post(const void* src, void* dst, size_t bytes, const unsigned long long* flags, int n_flags,
                 int* counter, void* stream);
/* Wait until flags[0..n_flags) (device ints of this rank that peers post to)
 * all reach e = *counter + 1, then advance *counter.  Gives up after about
 * one second: std_get_device_error then reports a wait timeout. */
int std_p2p_wait(const int* flags, int n_flags, int* counter, void* stream);
/* std_merge_partials_f32 with part i at parts[i] (n_parts <= 8 pointers, on
 * any GPU of the node): the same arithmetic, byte-identical results. */
int std_merge_partials_f32_list(const unsigned long long* parts, int n_parts, int rows, int D, void* out,
                                float* lse_out, void* stream);

/* ---- (f) verification-guided re-selection: the collector ------------- */

/* Replaces: RuntimeVerificationCollector._hook (dynamic_selection.py:290-308).
 * For the nq verify rows of one layer's dense forward: q_kv[t] = fp32 mean of
 * the G = Hq/Hkv query heads of each KV group (q [B, nq, Hq, D] bf16, after
 * RoPE), l[t, v] = q_kv[t] . k[visual_pos[v]] / sqrt(D) over the layer's K
 * cache k_cache [B, Hkv, cap, D], and rel_out[b][h][visual_pos[v]] =
 * sum_t softmax over v of l[t, :] (fp32; rel_out rows of rel_stride floats,
 * positions outside visual_pos untouched).  D = 128, nq <= 32. */
size_t std_collect_workspace_bytes(int B, int Hkv, int nq, int V);
int std_collect_relevance(const void* q, const void* k_cache, const int32_t* visual_pos, int V, int B, int nq, int Hq,
                          int Hkv, int D, int cap, float* rel_out, long long rel_stride, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ---- GEMM tuning and plan --------------------------------------------- */

/* Tuning (no reference counterpart): the per-CTA shared-memory budget of the
 * GEMMs' stage ring, 40..200 KiB (default 104 KiB, two CTAs per SM).
 * Applies to launches issued after the call, process-wide. */
int std_gemm_set_smem_budget(int bytes);
/* Launch plan (no reference counterpart): how many ranges K is split into
 * for a GEMM on an [N, K] weight matrix (split partials are summed in split
 * order by the epilogue kernel). */
int std_gemm_plan(int N, int K, int* splits_out);

/* ---- (d) fused greedy acceptance + rollback ---------------------------- */

/* Replaces: std_qwen25vl.py:806-815 (argmax compare, accepted prefix, bonus),
 * :910-921 (commit, EOS, max_new_tokens), :923-929 (dense/sparse cache length
 * rollback) and :931-939 (pending bonus).  Device state, int32 per request:
 * tok [B, tok_stride] (tok[0] pending bonus, tok[1..gamma] drafts), vpred
 * [B, vstride] verify-row argmax, dense_next [B] prefill argmax, ctx_len,
 * dense_len, sparse_len, n_gen, done [B], out_tokens [B, max_new], stats
 * [B, 4] (rounds, accepted, proposed, last accept), accept_hist [B, hist_cap]
 * (may be NULL).  pending = 1 when tok[0] holds a pending bonus (every round
 * after the first). */
int std_accept_commit(int B, int gamma, int pending, int32_t* tok, int tok_stride, const int32_t* vpred, int vstride,
                      const int32_t* dense_next, int max_new, int eos, int ignore_eos, int32_t* ctx_len,
                      int32_t* dense_len, int32_t* sparse_len, int32_t* n_gen, int32_t* done, int32_t* out_tokens,
                      int32_t* stats, int32_t* accept_hist, int hist_cap, void* stream);

/* Replaces: the verification policies of a parallel verify
 * (std_qwen25vl.py:816-884 margin check, math_on_full_accept and
 * verify_fallback; verification_policy.py:29-67 min_prediction_margin and
 * needs_sequential_fallback).  One thread per request (B <= 1024): computes
 * the accepted prefix, the smallest top-1 minus top-2 margin of the committed
 * predictions from margins [B, vstride] (threshold NaN: no margin check;
 * margin_hist [B, hist_cap] gets the round's value at index stats[b][0], NaN
 * when no prediction has a verify row), and whether the round is re-verified:
 * mode 0 none, 1 sequential_on_reject, 2 sequential_on_low_accept (accept <=
 * max_accept), 3 sequential_on_low_margin, 4 sequential_guard;
 * math_on_full_accept re-verifies a full accept.  rerun[b] (int32), counters
 * [B, 3] (+= margin reruns, fallbacks, accepted extra), first_accept [B],
 * any_rerun [1]; with cond != 0 (a conditional handle of the graph being
 * captured) the kernel also sets that IF condition to any_rerun.  after = 1:
 * the bookkeeping after a replay (accepted extra from the replayed vpred). */
int std_verify_policy(int B, int gamma, int pending, const int32_t* tok, int tok_stride, const int32_t* vpred,
                      int vstride, const int32_t* dense_next, int max_new, const int32_t* n_gen, const int32_t* done,
                      const int32_t* stats, const float* margins, float threshold, int mode, int max_accept,
                      int math_on_full_accept, int32_t* rerun, int32_t* first_accept, int32_t* counters,
                      float* margin_hist, int hist_cap, int32_t* any_rerun, unsigned long long cond, int after,
                      void* stream);

/* AR bookkeeping (std_qwen25vl.py:584-590).  std_ar_commit records
 * tok[b][0] as the next generated token of each running request and sets
 * active[b]; the step's forward writes its argmax to next_tok[b];
 * std_ar_advance then, for active requests, advances dense_len and ctx_len by
 * one and moves next_tok[b] into tok[b][0].  Finished requests stay frozen. */
int std_ar_commit(int B, int tok_stride, int max_new, int eos, int ignore_eos, const int32_t* tok, int32_t* n_gen,
                  int32_t* done, int32_t* out_tokens, int32_t* active, void* stream);
int std_ar_advance(int B, const int32_t* active, const int32_t* next_tok, int32_t* tok, int tok_stride,
                   int32_t* dense_len, int32_t* ctx_len, void* stream);

/* ---- (d) device-side decode loop (CUDA graph WHILE node) --------------- */

/* Replaces: the host-driven decode loops of std_qwen25vl.py:766-939 (STD
 * rounds, `while len(generated) < max_new_tokens`, with .tolist() host reads
 * each round) and :575-606 (AR steps).  Called while `stream` is capturing a
 * CUDA graph: enqueues a kernel that zeroes *counter and sets the loop
 * condition to "some done[b] == 0" (b < B), appends a WHILE conditional node,
 * and begins capturing `body_stream` (a different stream, not capturing) into
 * the node's body graph.  The caller then enqueues one loop iteration on
 * body_stream and calls std_capture_while_end, which enqueues the condition
 * update (counter += 1; continue while some request runs and counter <
 * max_iters) and ends the body capture.  handle_out receives the conditional
 * handle for std_capture_while_end, body_graph_out (optional) the body graph
 * (owned by the WHILE node).  done and counter are device int32. */
int std_capture_while_begin(void* stream, void* body_stream, const int32_t* done, int B, int32_t* counter,
                            unsigned long long* handle_out, void** body_graph_out);
int std_capture_while_end(void* body_stream, unsigned long long handle, const int32_t* done, int B, int32_t* counter,
                          int max_iters);
/* IF conditional node (no reference counterpart; it runs the re-verification
 * of std_verify_policy without a host round trip): std_graph_cond_handle
 * creates a handle in the graph `stream` is capturing, for the kernel that
 * sets it; std_capture_if_begin appends an IF node on that handle after the
 * stream's captured work and starts capturing body_stream into its body;
 * std_capture_if_end ends the body capture. */
int std_graph_cond_handle(void* stream, unsigned long long* handle_out);
int std_capture_if_begin(void* stream, void* body_stream, unsigned long long handle);
int std_capture_if_end(void* body_stream);
/* A new non-blocking CUDA stream on the current device, for capturing
 * conditional bodies (a stream distinct from every pooled stream). */
int std_stream_create(void** stream_out);
/* Launch accounting (no reference counterpart): how many kernel launches
 * this library has enqueued in this process so far, counting launches
 * recorded into CUDA graphs under stream capture.  Host-side counter. */
long long std_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* STD_B200_H */
