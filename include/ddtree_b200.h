/*
 * ddtree_b200 — C ABI of the B200 (sm_100a) DDTree verification hot path.
 *
 * All entry points take raw device pointers, sizes/strides and a cudaStream_t (passed
 * as void*), launch asynchronously on that stream, never allocate, never synchronise
 * the host, and return 0 or a negative DDT_ERR_* code.  Buffers (outputs and the
 * workspaces sized by the *_workspace_bytes queries) are owned by the caller.
 * Entry points are stateless and reentrant; concurrent calls must use distinct
 * workspaces.
 *
 * Reference interfaces replaced (paths are files of the DDTree research code):
 *   ddt_topk_tree        ddtree.py:84-166  build_ddtree_tree (fp32 topk + logsumexp,
 *                        best-first heap, visibility) fused with ddtree.py:227-267
 *                        compile_ddtree_tree (verify ids / positions); the visibility
 *                        matrix becomes per-node ancestor bitmasks
 *   ddt_argmax           model/utils.py:28-30  sample() at temperature 0
 *                        (torch.argmax over [N, V] logits, ddtree.py:478)
 *   ddt_accept_compact   ddtree.py:270-281 follow_verified_tree fused with
 *                        ddtree.py:284-335 compact_dynamic_cache
 *   ddt_compact_kv       ddtree.py:31-58 compact_tail_inplace (inline C++ extension)
 *                        applied to every layer's K and V in one launch
 *   ddt_tree_attn        transformers/integrations/sdpa_attention.py:40-103
 *                        (scaled_dot_product_attention with the additive tree mask of
 *                        ddtree.py:262-264), reached from the verify forward at
 *                        ddtree.py:467 through transformers' attention registry
 *   ddt_attn_merge       no reference counterpart: merges split-KV partial results
 *                        (within one GPU, and across GPUs after an NCCL exchange)
 *   ddt_mask_to_bits     ddtree.py:262-264 read backwards: additive mask block ->
 *                        ancestor bitmasks, for callers that only hold the mask
 *   ddt_lm_head_argmax   the verify forward's lm_head (ddtree.py:467-478) fused with
 *                        sample() at temperature 0 (model/utils.py:28-30)
 *   ddt_sample_chains    mdflash.py:19-40 sample_candidate_chains
 *   ddt_chain_tree       ddtree.py:169-224 build_sampled_candidate_tree
 */
#ifndef DDTREE_B200_H_
#define DDTREE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define DDT_OK 0
#define DDT_ERR_INVALID (-1)   /* bad argument: null pointer, negative size, bad stride */
#define DDT_ERR_CAPACITY (-2)  /* exceeds a compiled limit (budget, depth, nodes, ...) */
#define DDT_ERR_DTYPE (-3)     /* unsupported element type */
#define DDT_ERR_ALIGN (-4)     /* pointer or stride misaligned for vector / TMA access */
#define DDT_ERR_CUDA (-5)      /* CUDA runtime / launch error */
#define DDT_ERR_TIMEOUT (-6)   /* a bounded device-side wait expired (status word) */
#define DDT_ERR_WORKSPACE (-7) /* workspace too small */
#define DDT_ERR_SCRATCH_LIMIT (-8) /* needs more than the fixed no-alloc scratch array */

/* element types */
#define DDT_F32 0
#define DDT_BF16 1

/* compiled limits */
#define DDT_MAX_BUDGET 1024 /* tree nodes excluding the root */
#define DDT_MAX_DEPTH 20    /* drafted depths (block_size - 1) */
#define DDT_MAX_NODES (DDT_MAX_BUDGET + 1)

const char* ddt_error_string(int code);
int ddt_version(void);

/* ---- tree construction --------------------------------------------------
 * draft_logits: [depths, vocab] (row stride `row_stride` elements), dtype DDT_F32 or
 * DDT_BF16.  k = min(budget, vocab).  Outputs (device):
 *   top_log_probs f32 [depths, k], top_token_ids i64 [depths, k]   (may be NULL)
 *   node_token_ids i64 [budget], node_depths i64 [budget], parents i32 [budget + 1]
 *   node_count i32 [1]
 *   anc_bits u32 [budget + 1, anc_words]  (bit j of row i: node j is an ancestor-or-self
 *                                          of node i; anc_words >= ceil((budget+1)/32))
 *   verify_ids i64 [budget + 1], verify_pos i64 [budget + 1]  (may be NULL; root token
 *   read from root_token (device i64), positions start + depth)
 * The workspace must be zero-filled before its first use; every launch leaves its
 * counters at zero again. */
size_t ddt_topk_tree_workspace_bytes(int64_t depths, int64_t vocab, int64_t budget);
int ddt_topk_tree(const void* draft_logits, int dtype, int64_t depths, int64_t vocab,
                  int64_t row_stride, int64_t budget, float* top_log_probs,
                  int64_t* top_token_ids, int64_t* node_token_ids, int64_t* node_depths,
                  int32_t* parents, int32_t* node_count, uint32_t* anc_bits,
                  int64_t anc_words, const int64_t* root_token, int64_t start,
                  int64_t* verify_ids, int64_t* verify_pos, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Batched tree build: the trees of n_requests independent requests (the same depths and
 * vocabulary) in one launch, each exactly what ddt_topk_tree gives for that request.  No
 * counterpart in the reference, which builds one tree per ddtree_generate call
 * (ddtree.py:440); it serves a server that verifies many requests per step.
 *   draft_logits: request r, depth d at draft_logits + r * request_stride + d * row_stride
 *   budgets: i32 [n_requests] on the device, each in [0, max_budget] (larger values are
 *     clamped to max_budget; 0 gives the root-only tree)
 *   outputs per request at fixed strides: node_token_ids / node_depths [n_requests,
 *     max_budget]; parents / verify_ids / verify_pos [n_requests, max_budget + 1];
 *     anc_bits [n_requests, max_budget + 1, anc_words]; node_count i32 [n_requests]
 *   root_tokens i64 [n_requests] (may be NULL: root token 0), starts i64 [n_requests]
 *     (may be NULL: every start 0); verify_ids / verify_pos may be NULL
 * The workspace (ddt_topk_tree_batched_workspace_bytes) needs no initialisation: the call
 * zero-fills its per-request tickets (one cudaMemsetAsync on the stream) before the launch. */
size_t ddt_topk_tree_batched_workspace_bytes(int64_t n_requests, int64_t depths, int64_t vocab,
                                             int64_t max_budget);
int ddt_topk_tree_batched(const void* draft_logits, int dtype, int64_t n_requests,
                          int64_t depths, int64_t vocab, int64_t row_stride,
                          int64_t request_stride, const int32_t* budgets, int64_t max_budget,
                          int64_t* node_token_ids, int64_t* node_depths, int32_t* parents,
                          int32_t* node_count, uint32_t* anc_bits, int64_t anc_words,
                          const int64_t* root_tokens, const int64_t* starts,
                          int64_t* verify_ids, int64_t* verify_pos, void* workspace,
                          size_t workspace_bytes, void* stream);

/* Tree build that allocates nothing and takes no workspace.  No counterpart in the
 * reference: it serves callers that cannot allocate device memory when they call (a
 * serving stack that owns all device memory in its own pool after start-up, or a plugin
 * interface that passes only inputs and outputs).  Arguments and outputs are those of
 * ddt_topk_tree.  Scratch lives in a DDT_NOALLOC_SCRATCH_BYTES array inside the library's
 * device image, held by every GPU that loads the library until the process exits; its
 * address is looked up on a device's first call (make that call before any stream
 * capture), and again on the first call after the device's context was replaced
 * (cudaDeviceReset).  Problems whose workspace (ddt_topk_tree_workspace_bytes) exceeds the array
 * return DDT_ERR_SCRATCH_LIMIT: 15 depths x 151936 vocabulary fit up to budget 1024.
 * All calls share the array, so calls that overlap on the GPU race. */
#define DDT_NOALLOC_SCRATCH_BYTES (2u << 20)
int ddt_topk_tree_noalloc(const void* draft_logits, int dtype, int64_t depths, int64_t vocab,
                          int64_t row_stride, int64_t budget, float* top_log_probs,
                          int64_t* top_token_ids, int64_t* node_token_ids,
                          int64_t* node_depths, int32_t* parents, int32_t* node_count,
                          uint32_t* anc_bits, int64_t anc_words, const int64_t* root_token,
                          int64_t start, int64_t* verify_ids, int64_t* verify_pos,
                          void* stream);

/* ---- sampled draft trees (MDFlash / P-Express variants) ---------------------
 * ddt_sample_chains: chains i64 [num_samples, depths] (row-major); chain s holds sample s of
 * every depth, drawn with replacement from softmax(draft_logits[d] / temperature) by inverse
 * CDF with counter-based uniforms of (seed, offset, depth, sample), or, for temperature
 * < 1e-5, the depth's argmax (ties to the lowest index) for every sample.  Logits must be
 * finite.  Replaces sample_candidate_chains (mdflash.py:19-40); the draws follow the same
 * distribution as torch.multinomial, not its random stream.
 * ddt_chain_tree: the trie of the chains (chain stride in elements) with at most budget
 * nodes, in the reference's node order, written like ddt_topk_tree's outputs (node tokens,
 * depths, parents, node_count, ancestor bitmasks, verify ids / positions).  Replaces
 * build_sampled_candidate_tree (ddtree.py:169-224).  num_chains <= DDT_MAX_BUDGET. */
int ddt_sample_chains(const void* draft_logits, int dtype, int64_t depths, int64_t vocab,
                      int64_t row_stride, int64_t num_samples, float temperature, uint64_t seed,
                      uint64_t offset, int64_t* chains, void* stream);
int ddt_chain_tree(const int64_t* chains, int64_t num_chains, int64_t depths,
                   int64_t chain_stride, int64_t budget, int64_t* node_token_ids,
                   int64_t* node_depths, int32_t* parents, int32_t* node_count,
                   uint32_t* anc_bits, int64_t anc_words, const int64_t* root_token,
                   int64_t start, int64_t* verify_ids, int64_t* verify_pos, void* stream);

/* ---- greedy posterior ---------------------------------------------------
 * logits [rows, cols] (row stride in elements) -> out i64 [rows]; ties go to the lowest
 * index, NaN counts as the largest value. */
int ddt_argmax(const void* logits, int dtype, int64_t rows, int64_t cols, int64_t row_stride,
               int64_t* out, void* stream);

/* ---- fused lm_head -> greedy posterior ------------------------------------
 * out[n] = argmax_v bf16(hidden[n] . weight[v]) for n < n_rows (ties to the lowest index,
 * NaN largest), the logits being the bf16 rounding (nearest even) of fp32-accumulated dot
 * products; hidden [n_rows, hidden_size] and weight [vocab, hidden_size] bf16, row strides
 * hidden_ld / weight_ld elements, hidden_size a multiple of 64.  The [n_rows, vocab] logits
 * are not written unless logits_out (bf16, row stride logits_ld) is given, a testing aid.
 * Replaces the lm_head projection of the verify forward (ddtree.py:467-478) followed by
 * sample() at temperature 0 (model/utils.py:28-30).  The workspace
 * (ddt_lm_head_argmax_workspace_bytes) must be zero-filled before its first use; every
 * launch leaves it zeroed.  status: as for ddt_tree_attn. */
size_t ddt_lm_head_argmax_workspace_bytes(int64_t n_rows);
int ddt_lm_head_argmax(const void* hidden, int64_t hidden_ld, const void* weight,
                       int64_t weight_ld, int64_t n_rows, int64_t hidden_size, int64_t vocab,
                       int64_t* out, void* logits_out, int64_t logits_ld, void* workspace,
                       size_t workspace_bytes, int32_t* status, void* stream);

/* ---- accept walk + KV compaction ----------------------------------------
 * KV cache: n_tensors tensors (K and V of every layer) whose device base pointers are in
 * the DEVICE array kv_ptrs; each is [heads, seq, head_dim] with the given element
 * strides (head_dim contiguous), element size elem_bytes (2 or 4).  The tree window
 * starts at row past_length.
 * ddt_accept_compact: walks the tree from the root following posterior (i64 [n_nodes])
 * through parents / node_token_ids (node i >= 1 carries node_token_ids[i - 1]), writes
 * accepted (i64, capacity n_nodes), n_accepted (i32), next_token (i64), and moves cache
 * rows past_length + accepted[j] to past_length + j in every tensor.
 * ddt_compact_kv: the same move for a given keep list (device i64 [keep_count]). */
int ddt_accept_compact(const int64_t* posterior, const int32_t* parents,
                       const int64_t* node_token_ids, int64_t n_nodes, void* const* kv_ptrs,
                       int64_t n_tensors, int64_t heads, int64_t head_dim, int64_t head_stride,
                       int64_t seq_stride, int64_t elem_bytes, int64_t past_length,
                       int64_t* accepted, int32_t* n_accepted, int64_t* next_token,
                       void* stream);
int ddt_compact_kv(const int64_t* keep, int64_t keep_count, void* const* kv_ptrs,
                   int64_t n_tensors, int64_t heads, int64_t head_dim, int64_t head_stride,
                   int64_t seq_stride, int64_t elem_bytes, int64_t past_length, void* stream);
/* Batched walk + compaction: request r's tree (node_counts[r] + 1 nodes; parents,
 * node_token_ids and posterior rows at the given strides, as ddt_topk_tree_batched writes
 * them) is walked and its cache compacted exactly like ddt_accept_compact, all requests in one
 * launch.  kv_ptrs: device array [n_requests, n_tensors] of K/V bases; head_strides,
 * past_lengths: device i64 [n_requests] (a head stride that is not a whole number of 16-byte
 * vectors moves nothing and sets *status non-zero); outputs accepted [n_requests, acc_stride],
 * n_accepted i32 [n_requests], next_token i64 [n_requests].  No counterpart in the reference,
 * which compacts one request's cache per ddtree_generate round (ddtree.py:284-335). */
int ddt_accept_compact_batched(int64_t n_requests, const int64_t* posterior, int64_t post_stride,
                               const int32_t* parents, int64_t par_stride,
                               const int64_t* node_token_ids, int64_t ids_stride,
                               const int32_t* node_counts, int64_t max_nodes,
                               void* const* kv_ptrs, int64_t n_tensors, int64_t heads,
                               int64_t head_dim, const int64_t* head_strides, int64_t seq_stride,
                               int64_t elem_bytes, const int64_t* past_lengths, int64_t* accepted,
                               int64_t acc_stride, int32_t* n_accepted, int64_t* next_token,
                               int32_t* status, void* stream);

/* One decode-loop round's bookkeeping on the device, after the walk, for each request r
 * (one warp each), as ddtree.py:488-498 does on the host:
 *   output_ids[r, starts[r] + i] = verify_ids[r, accepted[r, i]]   for i < n_accepted[r]
 *   output_ids[r, starts[r] + n_accepted[r]] = next_token[r]
 *   root_tokens[r] = next_token[r]  (the next round's root, output_ids[start] there)
 *   acceptance[r, rounds[r]] = n_accepted[r]; rounds[r] += 1; starts[r] += n_accepted[r].
 * With it a recorded verify step advances its own device-side prefix length, so a host can
 * enqueue several rounds and sync once.  Writes at or beyond out_capacity / len_capacity
 * are dropped and set *status bit 8 (status may be null). */
int ddt_advance_round(int64_t n_requests, int64_t* starts, int32_t* rounds,
                      const int32_t* n_accepted, const int64_t* accepted, int64_t acc_stride,
                      const int64_t* verify_ids, int64_t ids_stride, int64_t max_nodes,
                      const int64_t* next_token, int64_t* root_tokens, int64_t* output_ids,
                      int64_t out_stride, int64_t out_capacity, int32_t* acceptance,
                      int64_t len_stride, int64_t len_capacity, int32_t* status, void* stream);

/* Row gather with a device-side count: out[i, :row_bytes] = src[idx[i], :row_bytes] for
 * i < min(*count, max_rows) (count may be null: max_rows rows); row strides in bytes; rows,
 * strides and both bases 16-byte aligned; an index outside [0, src_rows) gives a zero row.
 * Replaces the accepted-row gather of the target's context features,
 * extract_context_feature(...).index_select(1, accepted) (ddtree.py:487, model/utils.py:17-26),
 * without reading the accepted count on the host. */
int ddt_gather_rows(const void* src, int64_t src_rows, int64_t src_row_stride,
                    const int64_t* idx, const int32_t* count, int64_t max_rows, void* out,
                    int64_t out_row_stride, int64_t row_bytes, void* stream);

/* ---- tree attention -----------------------------------------------------
 * q: [n_nodes, q_heads, head_dim] bf16 at element strides (q_node_stride, q_head_stride);
 * k, v: [kv_heads, past_length + n_nodes, head_dim] bf16 at (kv_head_stride,
 * kv_seq_stride); out: [n_nodes, q_heads, head_dim] bf16 at (o_node_stride,
 * o_head_stride).  head_dim must be 128; q_heads a multiple of kv_heads.
 * mask_mode DDT_MASK_TREE: node i sees every prefix key and the tree keys of its
 * ancestors-or-self (anc_bits [n_nodes, anc_words]); DDT_MASK_CAUSAL: node i sees keys
 * < past_length + i + 1 (anc_bits unused); DDT_MASK_NONE: every query row sees every key
 * (anc_bits unused) -- the drafter's non-causal attention over context + block
 * (model/dflash.py:58-102, is_causal = False, no mask).
 * kv_splits: number of KV partitions per (head, query tile); 0 picks one.  Partial
 * results go to the workspace and are merged in the same call.
 * status: device i32 (zeroed by the caller), set non-zero if a bounded wait expired; the
 * output is then incomplete, and a caller that reads the status (after its own sync) reports
 * DDT_ERR_TIMEOUT. */
#define DDT_MASK_TREE 0
#define DDT_MASK_CAUSAL 1
#define DDT_MASK_NONE 2
size_t ddt_tree_attn_workspace_bytes(int64_t n_nodes, int64_t q_heads, int64_t head_dim,
                                     int64_t kv_splits);
int ddt_tree_attn(const void* q, int64_t q_node_stride, int64_t q_head_stride, const void* k,
                  const void* v, int64_t kv_head_stride, int64_t kv_seq_stride, void* out,
                  int64_t o_node_stride, int64_t o_head_stride, int64_t n_nodes,
                  int64_t past_length, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                  const uint32_t* anc_bits, int64_t anc_words, int mask_mode, float scale,
                  int64_t kv_splits, void* workspace, size_t workspace_bytes, int32_t* status,
                  void* stream);

/* ddt_tree_attn with the prefix length in device memory: *past_length_dev (i64, 8-byte
 * aligned) is read when the kernel runs, so that one launch recorded in a CUDA graph serves
 * every prefix length up to max_past_length (a decode loop whose prefix grows every round).
 * k, v: [kv_heads, max_past_length + n_nodes, head_dim] views; the tree's rows sit at
 * [live, live + n_nodes) and every key after them is masked.  The plan is the one of
 * ddt_tree_attn at max_past_length, and so is the cost.  mask_mode DDT_MASK_TREE or
 * DDT_MASK_CAUSAL; status is required: a live length outside [0, max_past_length] sets bit
 * 4 (the launch then runs at max_past_length, in bounds, and its output is not meaningful),
 * an expired wait bit 1.  Replaces the same call as ddt_tree_attn (sdpa_attention.py:92 via
 * ddtree.py:467), where the reference's prefix length is host state. */
int ddt_tree_attn_device_past(const void* q, int64_t q_node_stride, int64_t q_head_stride,
                              const void* k, const void* v, int64_t kv_head_stride,
                              int64_t kv_seq_stride, void* out, int64_t o_node_stride,
                              int64_t o_head_stride, int64_t n_nodes, int64_t max_past_length,
                              const int64_t* past_length_dev, int64_t q_heads, int64_t kv_heads,
                              int64_t head_dim, const uint32_t* anc_bits, int64_t anc_words,
                              int mask_mode, float scale, int64_t kv_splits, void* workspace,
                              size_t workspace_bytes, int32_t* status, void* stream);

/* Host-only query of the launch plan ddt_tree_attn uses for these sizes (key_end < 0, e.g.
 * -1), or ddt_tree_attn_partial_merged for the key shard [key_begin, key_end) (key_end >= 0;
 * an empty shard [b, b) included), computed by the same host function those entry points
 * launch through (no device work):
 * plan[0] = 1 for the balanced schedule (key tiles cut over the SMs by a cost model, parts
 * merged by a second kernel), 0 for uniform key splits; plan[1] = CTAs; plan[2] = partial
 * parts merged by a second kernel (0: none, one launch); plan[3] = the most work items one
 * CTA runs.  Returns 0, a DDT_ERR_* code for sizes the entry points reject, or 1 if the
 * balanced table fails its own consistency check (each key tile of each unit in exactly one
 * item).  An inspection aid for sizing and tests; it has no counterpart in the reference. */
int ddt_tree_attn_plan(int64_t n_nodes, int64_t past_length, int64_t q_heads, int64_t kv_heads,
                       int64_t kv_splits, int64_t key_begin, int64_t key_end, int64_t* plan);

/* Partial-result attention: like ddt_tree_attn but writes un-normalised fp32 partials over
 * the key range [key_begin, key_end) of this shard, for a cross-GPU split-KV merge, split
 * in-GPU into kv_splits key ranges (0 picks one; query ddt_tree_attn_partial_splits):
 * o_part [kv_splits, n_nodes * q_heads, head_dim], row max m and row sum l
 * [kv_splits, n_nodes * q_heads] (m in log2 units of the scaled scores).
 * Keys are indexed globally: this shard's k/v pointers address key key_begin. */
int64_t ddt_tree_attn_partial_splits(int64_t n_nodes, int64_t key_count, int64_t q_heads,
                                     int64_t kv_heads);
int ddt_tree_attn_partial(const void* q, int64_t q_node_stride, int64_t q_head_stride,
                          const void* k, const void* v, int64_t kv_head_stride,
                          int64_t kv_seq_stride, int64_t key_begin, int64_t key_end,
                          float* o_part, float* m_part, float* l_part, int64_t n_nodes,
                          int64_t past_length, int64_t q_heads, int64_t kv_heads,
                          int64_t head_dim, const uint32_t* anc_bits, int64_t anc_words,
                          int mask_mode, float scale, int64_t kv_splits, int32_t* status,
                          void* stream);

/* Like ddt_tree_attn_partial, but the shard's key tiles are spread evenly over the SMs
 * (balanced work items) and merged in-GPU, so the result is one partial per row:
 * o_part [n_nodes * q_heads, head_dim], m_part / l_part [n_nodes * q_heads].  Halves the
 * bytes a cross-GPU exchange moves against two in-GPU splits.  Needs a workspace of
 * ddt_tree_attn_partial_merged_workspace_bytes bytes (16-byte aligned).  Replaces, like
 * ddt_tree_attn_partial, one key shard of the verify attention of
 * integrations/sdpa_attention.py:40-103. */
size_t ddt_tree_attn_partial_merged_workspace_bytes(int64_t n_nodes, int64_t q_heads,
                                                    int64_t head_dim);
int ddt_tree_attn_partial_merged(const void* q, int64_t q_node_stride, int64_t q_head_stride,
                                 const void* k, const void* v, int64_t kv_head_stride,
                                 int64_t kv_seq_stride, int64_t key_begin, int64_t key_end,
                                 float* o_part, float* m_part, float* l_part, int64_t n_nodes,
                                 int64_t past_length, int64_t q_heads, int64_t kv_heads,
                                 int64_t head_dim, const uint32_t* anc_bits, int64_t anc_words,
                                 int mask_mode, float scale, void* workspace,
                                 size_t workspace_bytes, int32_t* status, void* stream);

/* Check of the bounded waits of the tree-attention kernel; no counterpart in the reference.
 * Every wait of that kernel gives up after a time limit (2 s in the entry points above),
 * sets the caller's status word, frees the kernel's tensor memory and lets the CTA return,
 * so a lost arrival cannot hang the GPU.  This launches the kernel once (tree mask, q
 * [n_nodes, q_heads, 128], k / v [kv_heads, past_length + n_nodes, 128], out like q, all
 * contiguous bf16) with its load-issuing warp withholding every load, so each consumer's
 * first wait runs out after timeout_ns (100 us .. 2 s).  The kernel must return and leave
 * *status (device i32, zeroed by the caller) non-zero; `out` holds zeros for the rows the
 * kernel reached.  Returns 0 when the launch was issued. */
int ddt_tree_attn_wait_check(const void* q, const void* k, const void* v, void* out,
                             int64_t n_nodes, int64_t past_length, int64_t q_heads,
                             int64_t kv_heads, const uint32_t* anc_bits, int64_t anc_words,
                             uint64_t timeout_ns, int32_t* status, void* stream);

/* Merge n_parts partials laid out [n_parts, rows, head_dim] / [n_parts, rows]
 * (rows = n_nodes * q_heads) into out (bf16, [n_nodes, q_heads, head_dim] at the given
 * strides). */
int ddt_attn_merge(const float* o_parts, const float* m_parts, const float* l_parts,
                   int64_t n_parts, int64_t n_nodes, int64_t q_heads, int64_t head_dim,
                   void* out, int64_t o_node_stride, int64_t o_head_stride, void* stream);

/* ---- split-KV exchange over NVLink peer memory (one node, up to 8 ranks) --------------
 * No counterpart in the reference.  Replaces the NCCL all-gather of the ranks' partials:
 * every rank allocates one receive buffer (ddt_peer_alloc: cudaMalloc, zeroed, and its
 * 64-byte CUDA IPC handle), the handles are exchanged over the process group, and every rank
 * opens the others' (ddt_peer_open).  Per call (epoch e = 1, 2, ..., the same on all ranks):
 * ddt_peer_push writes this rank's partial (O fp32 [rows, 128], m, l; rows = n_nodes *
 * q_heads) into slot `rank` of every buffer (peer_bases: host array of world pointers, this
 * rank's own buffer at index rank) and then bumps counter `rank` of each; ticket is a device
 * u32, zero before the first call, that every push leaves at zero.  ddt_peer_merge waits until
 * every rank's counter in the local buffer has reached e (bounded by timeout_ns, 100 us to
 * 2 s; on expiry it sets *status non-zero and the output is incomplete), then merges the world
 * partials like ddt_attn_merge.  Two parities of the buffer alternate between calls. */
size_t ddt_peer_buffer_bytes(int64_t world, int64_t n_nodes, int64_t q_heads, int64_t head_dim);
/* ddt_tree_attn_partial_merged and ddt_peer_push in one call: this rank's shard attention,
 * whose merge of the shard's key splits (when K / V exceed L2, the uniform-split plan) stores
 * the merged partial straight into every rank's receive buffer and bumps the counters; other
 * plans merge into the workspace and push with a copy kernel.  Workspace:
 * ddt_tree_attn_partial_push_workspace_bytes. */
size_t ddt_tree_attn_partial_push_workspace_bytes(int64_t n_nodes, int64_t q_heads,
                                                  int64_t head_dim);
int ddt_tree_attn_partial_push(const void* q, int64_t q_node_stride, int64_t q_head_stride,
                               const void* k, const void* v, int64_t kv_head_stride,
                               int64_t kv_seq_stride, int64_t key_begin, int64_t key_end,
                               int64_t n_nodes, int64_t past_length, int64_t q_heads,
                               int64_t kv_heads, int64_t head_dim, const uint32_t* anc_bits,
                               int64_t anc_words, int mask_mode, float scale,
                               void* const* peer_bases, int64_t world, int64_t rank,
                               uint32_t epoch, uint32_t* ticket, void* workspace,
                               size_t workspace_bytes, int32_t* status, void* stream);
int ddt_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int ddt_peer_open(const void* ipc_handle, void** ptr);
int ddt_peer_close(void* ptr);
int ddt_peer_free(void* ptr);
int ddt_peer_push(const float* o, const float* m, const float* l, int64_t n_nodes,
                  int64_t q_heads, int64_t head_dim, void* const* peer_bases, int64_t world,
                  int64_t rank, uint32_t epoch, uint32_t* ticket, void* stream);
int ddt_peer_merge(const void* local_base, int64_t world, int64_t n_nodes, int64_t q_heads,
                   int64_t head_dim, uint32_t epoch, void* out, int64_t o_node_stride,
                   int64_t o_head_stride, int32_t* status, uint64_t timeout_ns, void* stream);

/* ---- fused elementwise stages of the Qwen3 verify forward (bf16) ----------
 * ddt_add_rmsnorm: r = x + delta (delta may be NULL), writes r to residual_out (may be
 *   NULL, may alias x) and weight * rmsnorm(r) to norm_out; rows x hidden, hidden a
 *   multiple of 8 up to 16384.  Replaces the residual add of Qwen3DecoderLayer and
 *   Qwen3RMSNorm.forward (transformers/models/qwen3/modeling_qwen3.py:59-64).
 * ddt_qk_norm_rope_cache: from the fused projection qkv [n_tokens, (q_heads + 2 kv_heads),
 *   head_dim], applies q_norm / k_norm and the rotary embedding at positions (device i64),
 *   writes q to q_out [n_tokens, q_heads, head_dim] and k / v to rows past_length + i of the
 *   caches ([kv_heads, seq, head_dim] at the given strides).  Replaces
 *   modeling_qwen3.py:263-271 (q/k norm, apply_rotary_pos_emb :151-181, cos / sin of
 *   Qwen3RotaryEmbedding :137-147) and DynamicLayer.update (cache_utils.py:102-121).
 * ddt_rope_table: the bf16 cos / sin of the rotary embedding at positions (device i64) for
 *   the head_dim / 2 frequencies inv_freq, times rope_scale (Qwen3RotaryEmbedding.forward,
 *   modeling_qwen3.py:137-147), as table[n_tokens, head_dim / 2] of 32-bit words
 *   (cos | sin << 16); table 16-byte aligned.  Built once per forward.
 * ddt_qk_norm_rope_cache_table: ddt_qk_norm_rope_cache with cos / sin read from that table
 *   (bit-identical results).
 * ddt_qk_norm_rope_cache_table_device_past: the table form with the prefix length read from
 *   device memory (*past_length_dev, i64, 8-byte aligned) when the kernel runs, so that a
 *   recorded verify step serves every prefix length; the caches must hold max_past_length +
 *   n_tokens rows, and a value outside [0, max_past_length] writes nothing (the step's
 *   ddt_tree_attn_device_past reports it).  No counterpart in the reference, whose cache
 *   length is host state (cache_utils.py:102-121).
 * ddt_silu_mul: out[r, i] = silu(gate_up[r, i]) * gate_up[r, inter + i]; Qwen3MLP.forward
 *   (modeling_qwen3.py:81-83) between its projections. */
int ddt_add_rmsnorm(const void* x, const void* delta, const void* weight, int64_t rows,
                    int64_t hidden, float eps, void* residual_out, void* norm_out, void* stream);
int ddt_qk_norm_rope_cache(const void* qkv, int64_t n_tokens, int64_t q_heads, int64_t kv_heads,
                           int64_t head_dim, const void* q_norm_w, const void* k_norm_w, float eps,
                           const int64_t* positions, const float* inv_freq, float rope_scale,
                           void* q_out, void* k_cache, void* v_cache, int64_t head_stride,
                           int64_t seq_stride, int64_t past_length, void* stream);
int ddt_rope_table(const int64_t* positions, int64_t n_tokens, const float* inv_freq,
                   int64_t head_dim, float rope_scale, void* table, void* stream);
int ddt_qk_norm_rope_cache_table(const void* qkv, int64_t n_tokens, int64_t q_heads,
                                 int64_t kv_heads, int64_t head_dim, const void* q_norm_w,
                                 const void* k_norm_w, float eps, const void* rope_table,
                                 void* q_out, void* k_cache, void* v_cache, int64_t head_stride,
                                 int64_t seq_stride, int64_t past_length, void* stream);
int ddt_qk_norm_rope_cache_table_device_past(const void* qkv, int64_t n_tokens, int64_t q_heads,
                                             int64_t kv_heads, int64_t head_dim,
                                             const void* q_norm_w, const void* k_norm_w,
                                             float eps, const void* rope_table, void* q_out,
                                             void* k_cache, void* v_cache, int64_t head_stride,
                                             int64_t seq_stride, int64_t max_past_length,
                                             const int64_t* past_length_dev, void* stream);
int ddt_silu_mul(const void* gate_up, int64_t rows, int64_t inter, void* out, void* stream);

/* additive mask block [n_nodes, n_nodes] (row stride in elements; 0 = visible) ->
 * anc_bits [n_nodes, anc_words]. */
int ddt_mask_to_bits(const void* mask, int dtype, int64_t n_nodes, int64_t row_stride,
                     uint32_t* anc_bits, int64_t anc_words, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* DDTREE_B200_H_ */
