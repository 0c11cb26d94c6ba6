/*
 * qw_b200.h — C ABI of libqw_b200.so, the sm_100a kernels of the Qwen3.5-MoE
 * block-verify path.
 *
 * Conventions (all entry points):
 *   - pointers are DEVICE pointers unless stated otherwise; sizes are element
 *     counts; every tensor is dense row-major in the shape given;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - the return value is a qw_status; on failure qw_last_error() returns a
 *     thread-local message.  Arguments are validated on the host before any
 *     launch; nothing is allocated, and no entry point synchronizes the stream;
 *   - outputs are written only through the output pointers named in each
 *     signature; inputs are never written (the engine entry points document the
 *     state banks they update in place).
 *
 * Each function names the reference interface it replaces (paths relative to the
 * reference checkout).  The seven operators of the reference's fused-ops adapter
 * ABI (model/qwen35_moe_dflash/fused/ops.py:24-123, implemented on the host by
 * reference/fused_ops.py:28-173) keep their argument meaning.
 */
#ifndef QW_B200_H
#define QW_B200_H

#include <stddef.h>
#include <stdint.h>

/* bfloat16 storage in structs: __nv_bfloat16 for CUDA code, its 16-bit pattern in C. */
#if defined(__CUDACC__)
#include <cuda_bf16.h>
typedef __nv_bfloat16 qw_bf16_t;
#else
typedef uint16_t qw_bf16_t;
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define QW_ABI_VERSION 1

enum qw_status {
  QW_OK = 0,
  QW_ERR_ARG = 1,          /* invalid shape / dtype / pointer (Python: ValueError) */
  QW_ERR_UNSUPPORTED = 2,  /* valid but outside this build's kernels */
  QW_ERR_CUDA = 3,         /* a CUDA runtime error */
  QW_ERR_TIMEOUT = 4       /* a bounded device wait expired */
};

enum qw_dtype { QW_F32 = 0, QW_F16 = 1, QW_BF16 = 2 };

#define QW_MAX_BLOCK 16 /* tokens per sequence in one block verify (GDN kernels) */
#define QW_MAX_SEQ 256  /* tokens per sequence in one forward: prefill chunks (taken by the
                           GDN kernels in sub-blocks of QW_MAX_BLOCK) */
#define QW_MAX_CONV 8   /* largest causal-conv kernel width */

/* Mirrors FUSED_OPS_ABI = 1 (model/qwen35_moe_dflash/fused/ops.py:21). */
int qw_abi_version(void);
/* Thread-local message of the last failing call on this host thread. */
const char* qw_last_error(void);

/* ------------------------------------------------------------------------------
 * The seven fused-ops roles (reference/fused_ops.py), dtype-preserving.
 * ---------------------------------------------------------------------------- */

/* rms_norm(x, gamma, eps) — reference/fused_ops.py:28-34.
 * y = cast_y(cast_x(x * rsqrt(mean(x^2) + eps)) * gamma), x [rows, dim].
 * y_dtype must equal x_dtype, or be QW_F32 when gamma is QW_F32. */
int qw_rms_norm(const void* x, int x_dtype, const void* gamma, int gamma_dtype, void* y,
                int y_dtype, int64_t rows, int64_t dim, float eps, void* stream);

/* conv_state_update(projected, history) — reference/fused_ops.py:37-47.
 * projected [B,S,C], history [B,C,K-1] -> new_history [B,C,K-1], padded [B,C,S+K-1]. */
int qw_conv_state_update(const void* projected, const void* history, void* new_history,
                         void* padded, int dtype, int64_t batch, int64_t seq,
                         int64_t channels, int64_t hist, void* stream);

/* causal_conv1d(padded, weight) — reference/fused_ops.py:50-56 (no SiLU).
 * padded [B,C,L], weight [C,1,K] -> out [B,L-K+1,C]. */
int qw_causal_conv1d(const void* padded, const void* weight, void* out, int dtype,
                     int64_t batch, int64_t channels, int64_t padded_len, int64_t kernel,
                     void* stream);

/* chunk_gated_delta_rule(...) — reference/fused_ops.py:59-107 (sequential recurrence).
 * q,k [B,S,H,Dk], v [B,S,H,Dv], g,beta [B,S,H] (in_dtype), state0 [B,H,Dk,Dv]
 * (state_dtype F32 or F16), eff_len int16 [B] in [0,S] -> core [B,S,H,Dv] (in_dtype),
 * state_out [B,H,Dk,Dv] (state_dtype).  Dk,Dv <= 256. */
int qw_gated_delta_rule(const void* q, const void* k, const void* v, const void* g,
                        const void* beta, int in_dtype, const void* state0, int state_dtype,
                        const int16_t* eff_len, void* core, void* state_out, int64_t batch,
                        int64_t seq, int64_t heads, int64_t dk, int64_t dv, int use_l2norm,
                        void* stream);

/* cache_update(key, value, new_key, new_value) — reference/fused_ops.py:110-124.
 * key/value [B,Hkv,T0,D] (may be NULL with t_old == 0), new [B,Hkv,T1,D]
 * -> out [B,Hkv,T0+T1,D]. */
int qw_cache_update(const void* key, const void* value, const void* new_key,
                    const void* new_value, void* out_key, void* out_value, int dtype,
                    int64_t batch, int64_t kv_heads, int64_t t_old, int64_t t_new,
                    int64_t dim, void* stream);

/* attention(q, k, v, query_start, scale) — reference/fused_ops.py:127-145.
 * Causal GQA: q [B,H,S,D], k,v [B,Hkv,T,D] with T = query_start + S -> out [B,H,S,D].
 * D in {32, 64, 128, 256}; bf16 or fp16; `workspace` holds qw_attn_workspace_bytes. */
int qw_attention(const void* q, const void* k, const void* v, void* out, int dtype,
                 int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq, int64_t total,
                 int64_t dim, int64_t query_start, float scale, void* workspace, void* stream);

/* Scratch (bytes) of qw_attention / qw_attn_paged for keys up to max_len. */
int64_t qw_attn_workspace_bytes(int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq,
                                int64_t dim, int64_t max_len);

/* qw_attention without a workspace argument.  No counterpart in the reference: it is
 * an addition for callers that cannot allocate device memory per call (a host runtime
 * that owns all device memory through its own pool, or a thread on which a cudaMalloc
 * would synchronise the device).  The split-K scratch is a fixed array of
 * QW_ATTN_NOALLOC_SCRATCH_BYTES in this library's device memory, held on every GPU that
 * loads the library until the process exits; shapes whose qw_attn_workspace_bytes
 * exceeds it are rejected with QW_ERR_ARG.  Nothing is allocated.  The first call on
 * a device looks up the array's device address (cudaGetSymbolAddress, with that device
 * current), so make that first call before any stream capture.  All calls on a device
 * share the one array: calls that overlap on the GPU (other streams, other host threads)
 * race and corrupt each other's results; serialise them.  Nothing in the array needs
 * clearing between calls.  Same arguments and results as qw_attention. */
#define QW_ATTN_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
int qw_attention_noalloc(const void* q, const void* k, const void* v, void* out, int dtype,
                         int64_t batch, int64_t heads, int64_t kv_heads, int64_t seq, int64_t total,
                         int64_t dim, int64_t query_start, float scale, void* stream);

/* moe(hidden, router_weight, gate_up, down, top_k) — reference/fused_ops.py:148-173.
 * Dense expert weights in the activation dtype (bf16 or f16): hidden [T,H],
 * router [E,H], gate_up [E,2I,H], down [E,H,I] -> out [T,H].  Selection repeats
 * torch.topk's CPU order exactly (ties included); topk_idx_out (int32 [T,k], may be
 * NULL) receives it.  H, I multiples of 16; `workspace` holds qw_moe_workspace_bytes. */
int qw_moe(const void* hidden, const void* router, const void* gate_up, const void* down,
           void* out, int dtype, int64_t tokens, int64_t hidden_dim, int64_t experts,
           int64_t inter, int64_t top_k, int32_t* topk_idx_out, void* workspace, void* stream);

/* Device scratch (bytes) the MoE entry points need for `tokens` routed tokens; the
 * caller allocates it (the library allocates nothing).  1 <= top_k <= 16: torch's
 * selection order is reproduced for sorts of up to 16 selected entries. */
int64_t qw_moe_workspace_bytes(int64_t tokens, int64_t hidden, int64_t experts, int64_t inter,
                               int64_t top_k);

/* ------------------------------------------------------------------------------
 * Weight streams.  A W4 stream packs int4 weights (symmetric, bf16 scale per group
 * of `group` along K) of an [N,K] matrix in the order the tensor-core fragments
 * consume them: per 16-row tile, per K group, 8*group bytes of nibbles followed by
 * 32 bytes of scales.  A B16 stream packs a bf16 [N,K] matrix the same way, per
 * 16-row tile and 64-wide K chunk (2048 bytes).  The packing is done by the Python
 * package (qwen35_dflash_b200.w4); these give the byte sizes.
 * Replaces the quantised-linear weight contract of
 * model/qwen35_moe_dflash/fused/quantization.py:154-165 (W4A8 g256 there).
 * ---------------------------------------------------------------------------- */
int64_t qw_w4_stream_bytes(int64_t n, int64_t k, int32_t group);
int64_t qw_b16_stream_bytes(int64_t n, int64_t k);

/* Output modes of the streaming linear kernels. */
enum qw_linear_mode {
  QW_OUT_BF16 = 0,      /* y[t,n] = bf16(acc) */
  QW_OUT_F32 = 1,       /* y[t,n] = acc */
  QW_OUT_RESID_BF16 = 2 /* y[t,n] = bf16(y[t,n] + bf16(acc)), in place (residual add) */
};

/* Quantised linear y = x . W^T with W a W4 stream — fused/quantization.py:154-165,
 * fused/model.py:197-204.  x bf16 [T,K], N % 16 == 0, K % group == 0,
 * group in {32,64,128}; y row stride ldy (elements). */
int qw_w4_linear(const void* x, const void* w_stream, void* y, int mode, int64_t ldy,
                 int64_t tokens, int64_t n, int64_t k, int32_t group, void* stream);

/* Dense bf16 linear y = x . W^T with W a B16 stream (router, GDN a/b predictors,
 * shared-expert gate) — fused/model.py:197-204.  K % 64 == 0. */
int qw_b16_linear(const void* x, const void* w_stream, void* y, int mode, int64_t ldy,
                  int64_t tokens, int64_t n, int64_t k, void* stream);

/* ------------------------------------------------------------------------------
 * W4A16 routed MoE, in three launches on one workspace — the quantized MoE chain of
 * model/qwen35_moe_dflash/fused/quantization.py:181-202 (gating top-k softmax ->
 * init routing -> grouped gate_up -> SwiGLU -> grouped down -> finalize routing),
 * with the reference's selection and rounding (reference/fused_ops.py:161-172) and
 * the shared expert of fused/model.py:305-307.
 * ---------------------------------------------------------------------------- */

/* Routing from router logits [T, ldl] (logit_dtype): fp32 softmax over the first
 * `experts` columns, torch.topk CPU order, renormalized weights cast to act_dtype;
 * column `shared_col` (or -1) holds the shared-expert gate logit.  Writes the top-k
 * indices and weights into the workspace; the per-expert (token, slot) lists are
 * built by the expert entry points (or qw_moe_route_lists). */
int qw_moe_route(const void* logits, int logit_dtype, int64_t ldl, int64_t tokens,
                 int64_t experts, int64_t top_k, int64_t shared_col, int act_dtype,
                 void* workspace, void* stream);

/* qw_moe_route that also stages the expert input x (bf16 [T, hidden], the x the next
 * expert call on this workspace receives; it must not change in between) for the
 * gate/up kernel: fp16 copy and per-group sums, written once per block instead of by
 * every gate/up CTA.  hidden and group as in that call; staged only for blocks of
 * <= 16 tokens with hidden a multiple of 256 and x 16-byte aligned (otherwise this is
 * qw_moe_route and the expert call converts x itself).  tie_order 1: qw_moe_route's
 * outputs exactly; 0: the same selected experts and weights, but experts whose logits
 * tie inside the top k may be listed in ascending id instead of torch.topk's order
 * (only a tie between the k-th and (k+1)-th logits runs the order emulation).  No
 * consumer of the routing depends on that order (the combine adds experts in
 * ascending id; equal weights renormalise to the same bits), so the MoE outputs are the
 * same bits.  No counterpart in the reference: qw_moe_route's extra work. */
int qw_moe_route_x(const void* logits, int logit_dtype, int64_t ldl, int64_t tokens,
                   int64_t experts, int64_t top_k, int64_t shared_col, int act_dtype,
                   const void* x, int64_t hidden, int32_t group, void* workspace, void* stream,
                   int32_t tie_order);

/* The per-expert lists of a routed block in the workspace: active experts in
 * ascending id, and for each its (token, slot) pairs in ascending token (the order in
 * which fused_ops.py:165-172 visits them). */
int qw_moe_route_lists(void* workspace, int64_t tokens, int64_t experts, int64_t top_k, void* stream);

/* Expert FFNs on the routing in `workspace`: x bf16 [T,H]; gate_up / down are W4
 * streams of [E][2I,H] / [E][H,I] (experts concatenated); the shared expert's
 * [2I,H] (gate rows then up rows) and [H,I] streams, or both NULL.  Writes each
 * (token, slot)'s raw fp32 expert output into the workspace. */
int qw_moe_experts_w4(const void* x, const void* gate_up, const void* down,
                      const void* shared_gate_up, const void* shared_down, int64_t tokens,
                      int64_t hidden, int64_t experts, int64_t inter, int64_t top_k,
                      int32_t group, void* workspace, void* stream);

/* Dense experts on the tensor cores.  With blocks of more than 16 tokens, a routed
 * expert that receives at least `tokens` (token, slot) pairs runs on the tcgen05
 * kernels (int4 expanded to 16-bit integers in shared memory, one fp32 tensor-memory
 * accumulator per quantisation group, scaled and summed in fp32) instead of the grouped
 * mma.sync kernels -- when such experts make at least 128 gate/up work items (tiles of
 * 128 pairs x 64-column blocks), decided on the device from the routing; group 128,
 * hidden and inter multiples of 128, not on the expert-parallel receiver.  Their outputs
 * then differ from the grouped kernels' in fp32 summation order only.  Process-wide;
 * 0 disables; default 0 (off: measured no faster than the grouped kernels on random,
 * Zipf(1.1) or 8-hot-expert routings); 128 is the tuned value when enabled.  Returns the
 * previous threshold (tokens < 0: query only).
 * The reference computes every expert with one grouped matmul
 * (quantization.py:181-202). */
int32_t qw_moe_dense_threshold(int32_t tokens);

/* The two halves of qw_moe_experts_w4 (same arguments), for timing each launch:
 * up = gate_up + SiLU*up into the workspace, down = down projection. */
int qw_moe_up_w4(const void* x, const void* gate_up, const void* down, const void* shared_gate_up,
                 const void* shared_down, int64_t tokens, int64_t hidden, int64_t experts,
                 int64_t inter, int64_t top_k, int32_t group, void* workspace, void* stream);
int qw_moe_down_w4(const void* x, const void* gate_up, const void* down, const void* shared_gate_up,
                   const void* shared_down, int64_t tokens, int64_t hidden, int64_t experts,
                   int64_t inter, int64_t top_k, int32_t group, void* workspace, void* stream);

/* qw_moe_experts_w4 for the routed experts [expert_lo, expert_lo + expert_count) of the
 * routing only (gate_up / down hold those experts' streams, indexed e - expert_lo; pairs
 * of other experts are left out, expert_count 0 computes only the shared expert).  The
 * expert-parallel building block; no counterpart in the reference. */
int qw_moe_experts_w4_range(const void* x, const void* gate_up, const void* down,
                            const void* shared_gate_up, const void* shared_down, int64_t tokens,
                            int64_t hidden, int64_t experts, int64_t inter, int64_t top_k,
                            int32_t group, int64_t expert_lo, int64_t expert_count, void* workspace,
                            void* stream);

/* ------------------------------------------------------------------------------
 * Expert parallelism: experts [g E/G, (g+1) E/G) live on rank g (one process per GPU);
 * attention, GDN and the shared expert stay with each rank's own requests.  The
 * reference shards the routed MoE of reference/fused_ops.py:148-173 (its quantised
 * chain model/qwen35_moe_dflash/fused/quantization.py:181-202) this way in its serving
 * plan; it has no multi-GPU code, so these entry points have no direct counterpart.
 *
 * The exchange is device-initiated over NVLink: each rank allocates one window of
 * qw_ep_window_bytes (qw_ep_window_alloc, which also returns its 64-byte IPC handle),
 * the ranks swap handles on the host once, and each maps its peers' windows
 * (qw_ep_window_open).  `peers` is then a device array of `ranks` uint64 window
 * addresses, this rank's own window at index `rank`.  Per MoE layer, after routing the
 * rank's `tokens` over all experts (qw_moe_route / qw_moe_route_x into `workspace`):
 *   qw_moe_ep_dispatch    each routed (token, slot) pair's row into its expert owner's
 *                         window (peer stores), then a release flag in every window;
 *   qw_moe_ep_recv_route  waits (bounded) for every rank's dispatch, routes the rows it
 *                         received (top-1 = their local expert) into a workspace of
 *                         qw_moe_ep_recv_workspace_bytes;
 *   qw_moe_ep_experts     this rank's experts over those rows (gate_up_local /
 *                         down_local: the streams of its experts only); the down
 *                         projection's epilogue stores the outputs, as bf16, into their
 *                         source ranks' windows and raises a release flag in every
 *                         window (the combine half of the exchange, inside the kernel);
 *   qw_moe_ep_scatter     waits (bounded) for every rank's results, writes the returned
 *                         rows into the routing's per-(token, slot) outputs for
 *                         qw_moe_combine(_norm), and closes the exchange -- or
 *   qw_moe_ep_combine_norm  does the combine + next RMSNorm reading the returned rows
 *                         directly (waits, then closes the exchange).
 * With shared = 1 the shared expert travels the same way: every rank holds it as local
 * expert E/G, after its routed experts (gate_up_local / down_local carry E/G + 1
 * experts), and each token sends it one more row, to its own rank.  local_experts =
 * E/G + shared; cap = tokens * (top_k + shared) (every rank the same tokens).  Every rank issues the same calls in
 * the same order; calls are stream-ordered (graph-capturable), and the results equal
 * the one-GPU MoE bit for bit.  A wait that expires (a lost peer) records
 * QW_ERR_TIMEOUT for qw_wait_status / qw_check_wait_status.
 * ---------------------------------------------------------------------------- */
int64_t qw_ep_window_bytes(int64_t ranks, int64_t cap, int64_t hidden);
/* The window's allocation (cudaMalloc, zeroed) and IPC handle: the only allocating
 * calls of the library, made once per engine. */
int qw_ep_window_alloc(int64_t bytes, void** window, void* ipc_handle);
int qw_ep_window_open(const void* ipc_handle, void** peer_window);
int qw_ep_window_close(void* peer_window);
int qw_ep_window_free(void* window);
int64_t qw_moe_ep_recv_workspace_bytes(int64_t ranks, int64_t cap, int64_t hidden, int64_t local_experts,
                                       int64_t inter);
int qw_moe_ep_dispatch(const void* workspace, const void* x, int64_t tokens, int64_t hidden,
                       int64_t experts, int64_t top_k, int64_t ranks, int64_t rank, int64_t cap,
                       int shared, const void* peers, void* window, void* stream);
int qw_moe_ep_recv_route(void* window, int64_t ranks, int64_t cap, int64_t hidden, int64_t local_experts,
                         void* recv_workspace, void* stream);
int qw_moe_ep_experts(void* window, const void* gate_up_local, const void* down_local, int64_t ranks,
                      int64_t rank, int64_t cap, int64_t hidden, int64_t local_experts, int64_t inter,
                      int32_t group, const void* peers, void* recv_workspace, void* stream);
int qw_moe_ep_scatter(void* workspace, void* window, int64_t tokens, int64_t hidden, int64_t experts,
                      int64_t inter, int64_t top_k, int64_t ranks, int64_t cap, int shared, void* stream);
/* qw_moe_combine_norm reading the expert outputs straight from the window (the returned
 * bf16 rows) instead of the workspace: waits (bounded) for every rank's results, then
 * closes the exchange (in place of qw_moe_ep_scatter + qw_moe_combine_norm). */
int qw_moe_ep_combine_norm(void* workspace, void* window, int64_t ranks, int64_t cap, void* hidden,
                           int64_t tokens, int64_t hidden_dim, int64_t experts, int64_t inter,
                           int64_t top_k, int has_shared, const void* gamma, void* normed, float eps,
                           void* tap, int64_t ldf, int tap_normed, void* stream);

/* Byte offset, inside a MoE workspace, of the int32 count of active routed experts
 * (valid after qw_moe_route_lists or an expert entry point; for measuring the experts
 * actually streamed). */
int32_t qw_moe_active_experts(const void* workspace, int64_t tokens, int64_t experts, int64_t top_k);

/* Weighted combine in ascending expert order (+ gated shared expert): out bf16 [T,H]
 * is overwritten, or, with residual != 0, out = bf16(out + moe) in place. */
int qw_moe_combine(void* workspace, void* out, int residual, int64_t tokens, int64_t hidden,
                   int64_t experts, int64_t inter, int64_t top_k, int has_shared, void* stream);

/* qw_moe_combine (residual form, bf16) fused with the RMSNorm that follows it at a
 * layer boundary (fused/model.py:386-409: the next layer's input norm, or the final
 * norm): hidden = bf16(hidden + moe) in place, then normed = rms_norm(hidden) with the
 * +1 gamma convention as qw_residual_norm, and, when tap != NULL, the feature tap
 * (hidden, or normed with tap_normed != 0) at tap[t*ldf + i].  hidden, normed, gamma
 * and tap 8-byte aligned, hidden_dim and ldf multiples of 4; top_k <= 16.  The kernel
 * reads hidden, gamma and the routing before it waits for the launch ahead of it (the
 * expert call), so that launch must not be the one that wrote hidden. */
int qw_moe_combine_norm(void* workspace, void* hidden, int64_t tokens, int64_t hidden_dim,
                        int64_t experts, int64_t inter, int64_t top_k, int has_shared,
                        const void* gamma, void* normed, float eps, void* tap, int64_t ldf,
                        int tap_normed, void* stream);

/* Host helper: device addresses of the routing results inside a workspace
 * (part fp32 [T,k+1,H], topk_idx int32 [T,k], topk_w fp32 [T,k], shared_gate fp32 [T]). */
int qw_moe_partials(void* workspace, int64_t tokens, int64_t hidden, int64_t experts,
                    int64_t inter, int64_t top_k, const float** part, const int32_t** topk_idx,
                    const float** topk_w, const float** shared_gate);

/* ------------------------------------------------------------------------------
 * Full-attention layer of the block verify (engine layer) — FusedTargetModel._attention
 * (model/qwen35_moe_dflash/fused/model.py:278-294) over a paged bf16 KV cache.
 * KV cache layout [pages, kv_heads, page_size, dim]; sequence b's position t is in
 * page pages[b*max_pages + t/page_size]; qpos[b] = tokens already cached before the
 * block (the block's first position).
 * ---------------------------------------------------------------------------- */

/* q/k RMSNorm (zero-centred weights, +1), partial RoPE on the first rotary_dim dims
 * (theta, fp32 angles), and the K/V append of the block (the CacheUpdate role,
 * reference/fused_ops.py:110-124).  qkv bf16 [B*S, ldq] holds per head [q | gate]
 * (heads*2*dim), then k (kv_heads*dim), then v.  q_out bf16 [B, heads, S, dim].  The
 * kernel reads the norm weights, qpos and the page table before it waits for the launch
 * ahead of it (the projection writing qkv), so that launch must not be the one that
 * wrote them. */
int qw_attn_prep(const void* qkv, int64_t ldq, const void* q_norm_w, const void* k_norm_w,
                 float eps, float rope_theta, int32_t rotary_dim, const int32_t* qpos,
                 const int32_t* pages, int32_t max_pages, int32_t page_size, void* k_cache,
                 void* v_cache, void* q_out, int64_t batch, int64_t seq, int64_t heads,
                 int64_t kv_heads, int64_t dim, void* stream);

/* Causal GQA of q [B,heads,S,dim] against the paged cache (keys <= qpos[b]+s), times
 * sigmoid(gate) (gate element (b,h,s,d) at gate + (b*S+s)*ldg + h*2*dim + d, or NULL),
 * -> out bf16 [B*S, heads*dim] (reference/fused_ops.py:127-145, fused/model.py:291-293).
 * max_len bounds qpos[b]+S over the batch and sizes the key splits. */
int qw_attn_paged(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                  int32_t max_pages, int32_t page_size, const int32_t* qpos, int64_t max_len,
                  const void* gate, int64_t ldg, void* out, int64_t batch, int64_t seq,
                  int64_t heads, int64_t kv_heads, int64_t dim, float scale, void* workspace,
                  void* stream);

/* ------------------------------------------------------------------------------
 * Gated-DeltaNet block verify and commit (engine layer).
 * One GDN layer's device buffers for a block of `seq` tokens of `batch` sequences;
 * token row t = b*seq + s.  The recurrent-state bank stores each head column-major,
 * [slots, v_heads, dv, dk]; `slots[b]` selects sequence b's row of both banks.
 * Replaces FusedTargetModel._gdn (model/qwen35_moe_dflash/fused/model.py:227-263)
 * with the operator sequence conv_state_update -> causal_conv1d -> SiLU ->
 * chunk_gated_delta_rule -> gated RMSNorm (reference/fused_ops.py:37-107).
 * ---------------------------------------------------------------------------- */
typedef struct {
  const qw_bf16_t* proj;     /* [T, ldp]: q | k | v conv channels, then z            */
  const float* ab;           /* [T, 2*v_heads]: in_proj_b logits, then in_proj_a      */
  qw_bf16_t* conv_hist;      /* [slots, channels, conv_k-1] conv tail bank            */
  const qw_bf16_t* conv_w;   /* [channels, conv_k]                                    */
  const float* A_log;        /* [v_heads]                                             */
  const float* dt_bias;      /* [v_heads]                                             */
  const qw_bf16_t* norm_w;   /* [dv] gated-norm weight (effective, no +1)             */
  float* state;              /* [slots, v_heads, dv, dk] recurrent-state bank         */
  qw_bf16_t* out;            /* [T, v_heads*dv] gated-norm output (verify only)       */
} qw_gdn_layer;

typedef struct {
  int32_t batch, seq, k_heads, v_heads, dk, dv, channels, conv_k, ldp;
  float eps;                 /* RMSNorm epsilon of the gated norm                    */
  const int32_t* slots;      /* device [batch]: bank row of each sequence             */
  const int32_t* accepted;   /* device [batch]: tokens to commit (commit only)        */
} qw_gdn_dims;

/* Block verify of one layer (`layers_dev[layer]`, a device array): writes out[],
 * reads the banks, never writes them.  (dk,dv) in {(128,128),(64,64),(128,64)},
 * 1 <= seq <= QW_MAX_SEQ (a block verify: seq <= QW_MAX_BLOCK; a prefill chunk may be
 * longer); proj 16-byte aligned with ldp a multiple of 8.  The kernel
 * reads proj, the banks and the conv weights, and runs the conv and the q/k norms,
 * before it waits for the launch ahead of it (the a/b projection, whose output `ab` it
 * reads after the wait), so that launch must not be the one that wrote proj. */
int qw_gdn_verify(const qw_gdn_dims* dims, const qw_gdn_layer* layers_dev, int layer,
                  void* stream);

/* Commit of `nlayers` layers (device array): the recurrent state and conv tail of
 * each sequence advance by accepted[b] tokens of the verified block, in place —
 * TargetVerification.commit (model/qwen35_moe_dflash/fused/session.py:374-387). */
int qw_gdn_commit(const qw_gdn_dims* dims, const qw_gdn_layer* layers_dev, int nlayers,
                  void* stream);

/* ------------------------------------------------------------------------------
 * Layer boundaries and the verify decision (engine layer).
 * ---------------------------------------------------------------------------- */

/* Residual-stream RMSNorm of FusedTargetModel._norm (fused/model.py:206-217) with a
 * zero-centred weight: normed = bf16(bf16(h*rsqrt(mean(h^2)+eps)) * bf16(gamma+1)).
 * With ids (int32 [T]) the stream is first set to embed[ids] (:346-347).  With tap,
 * the residual stream (or, tap_normed != 0, the normed output) is also copied to
 * tap[t*ldf + i] (the feature taps of :405-409). */
int qw_residual_norm(void* hidden, const int32_t* ids, const void* embed, const void* gamma,
                     void* normed, void* tap, int64_t ldf, int tap_normed, int64_t tokens,
                     int64_t hidden_dim, float eps, void* stream);

/* lm_head + argmax of fused/model.py:410-417: x bf16 [T,K] (T <= 16), W a B16 stream
 * of [N,K]; writes one (value, index) key per CTA and token into keys (u64
 * [qw_lmhead_blocks(N), T]) and, when logits != NULL, bf16 logits [T,N]. */
int64_t qw_lmhead_blocks(int64_t n);
int qw_lmhead_argmax(const void* x, const void* w_stream, void* logits, void* keys,
                     int64_t tokens, int64_t n, int64_t k, void* stream);

/* Acceptance of a verified block (fused/session.py:316-341, execution/runtime.py:83-95):
 * top1[t] = argmax of row t (ties -> lowest id); max_accepted[b] = longest prefix of
 * proposals[b*seq..] equal to (next_token[b], top1[b*seq], ...).  With auto_commit,
 * accepted[b] = max_accepted[b], next_token[b] = top1 of row accepted-1, qpos[b] +=
 * accepted (all device-side: no host synchronization).  One CTA per row; the last to
 * finish decides acceptance through a counter inside the library, so calls on one GPU
 * must not overlap. */
int qw_accept(const void* keys, int64_t nblk, const int32_t* proposals, int32_t* top1,
              int32_t* max_accepted, int32_t* next_token, int32_t* accepted, int32_t* qpos,
              int64_t batch, int64_t seq, int auto_commit, void* stream);

/* Commit bookkeeping for host-chosen accepted counts (TargetVerification.commit,
 * fused/session.py:374-387): next_token and qpos advance as in qw_accept. */
int qw_apply_commit(const int32_t* accepted, const int32_t* top1, int32_t* next_token,
                    int32_t* qpos, int64_t batch, int64_t seq, void* stream);

/* ------------------------------------------------------------------------------
 * The DFlash draft forward (model/qwen35_moe_dflash/model.py:102-522; block and context
 * of the draft graph model/qwen35_moe_dflash/reference/graphs.py:63-97).  Its
 * projections use qw_b16_linear, its norms qw_rms_norm (the draft stores effective
 * norm weights), its attention qw_attn_paged_masked.
 * ---------------------------------------------------------------------------- */

/* qw_attn_paged without the output gate and with the draft's masks: block_full = 1
 * lets every query row see the whole block (the draft's full-attention layer,
 * model.py:134-141), window > 0 hides keys at or beyond `window` positions before the
 * row (its sliding layers, model.py:170-175). */
int qw_attn_paged_masked(const void* q, const void* k_cache, const void* v_cache, const int32_t* pages,
                         int32_t max_pages, int32_t page_size, const int32_t* qpos, int64_t max_len,
                         void* out, int64_t batch, int64_t seq, int64_t heads, int64_t kv_heads,
                         int64_t dim, float scale, int block_full, int32_t window, void* workspace,
                         void* stream);

/* q/k RMSNorm with effective weights (ops.py:66-71), rotary over the whole head
 * (model.py:80-99, ops.py:75-90) and the append of k, v into the paged cache.  qkv rows
 * [B*S, ldq] hold [q (heads*dim, when has_q) | k | v]; row (b, s) sits at position
 * pos_base[b] - pos_sub[b] (pos_sub may be NULL) + s; with valid (int32 [B]) rows s >=
 * valid[b] are skipped (the context rows of a partly accepted block).  q goes to q_out
 * [B, heads, S, dim]. */
int qw_draft_prep(const void* qkv, int64_t ldq, int has_q, const void* q_norm_w, const void* k_norm_w,
                  float eps, float rope_theta, const int32_t* pos_base, const int32_t* pos_sub,
                  const int32_t* valid, const int32_t* pages, int32_t max_pages, int32_t page_size,
                  void* k_cache, void* v_cache, void* q_out, int64_t batch, int64_t seq, int64_t heads,
                  int64_t kv_heads, int64_t dim, void* stream);

/* out [T, inter] = bf16(bf16(silu(gate)) * up) from gate_up [T, 2 inter] = [gate | up]
 * (the draft MLP, model.py:265-291). */
int qw_swiglu(const void* gate_up, void* out, int64_t tokens, int64_t inter, void* stream);

/* hidden [B*S, H] = embed[anchor[b]] for s = 0, embed[mask_id] otherwise (graphs.py:74-86,
 * model.py:519-522 with the unit embedding scale). */
int qw_draft_block_embed(const void* embed, const int32_t* anchor, int32_t mask_id, void* hidden,
                         int64_t batch, int64_t seq, int64_t hidden_dim, void* stream);

/* The next verify block from the draft's lm_head keys (qw_lmhead_argmax): tokens[b*S] =
 * anchor[b], tokens[b*S + i] = stable arg-max of draft row i, i = 1 .. S-1
 * (graphs.py:87-97, model.py:496-517). */
int qw_draft_propose(const void* keys, int64_t nblk, const int32_t* anchor, int32_t* tokens,
                     int64_t batch, int64_t seq, void* stream);

/* ------------------------------------------------------------------------------
 * Bounded device waits.  Kernels that wait on the TMA engine (the cluster linears,
 * the bulk expert kernels) give up after a bounded time instead of hanging, record
 * the expiry in a sticky status word of the library and return early: the outputs of
 * that launch are then incomplete.  The reference fails fast on any backend error and
 * never retries or falls back (model/qwen35_moe_dflash/fused/ops.py:133-136); these
 * two calls are how that error reaches the host.
 * ---------------------------------------------------------------------------- */

/* Stream-ordered (graph-capturable) report: after every earlier kernel on the stream,
 * writes QW_OK or QW_ERR_TIMEOUT into status (int32, device) and, with clear != 0,
 * resets the sticky words. */
int qw_wait_status(int32_t* status, int clear, void* stream);

/* Synchronous check: synchronizes the stream, returns QW_ERR_TIMEOUT (with a message
 * naming the kernel family) if a wait expired since the last clear, else QW_OK; with
 * clear != 0 the sticky words are reset. */
int qw_check_wait_status(int clear, void* stream);

/* Test hook: every later cluster-linear launch from this process waits at most
 * limit_cycles (0 = the default of about a second) and announces tx_excess_bytes more
 * on each weight stage than it copies, so that its waits expire (no fault, no hang);
 * MoE expert launches take the limit only.  (0, 0) restores normal operation. */
int qw_debug_inject_wait_timeout(int64_t limit_cycles, int64_t tx_excess_bytes);

#ifdef __cplusplus
}
#endif

#endif /* QW_B200_H */
