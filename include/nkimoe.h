/*
 * nkimoe.h - C ABI of the B200 (sm_100a) implementation of the Qwen3-30B-A3B
 * sparse-MoE block and the norms that feed it.
 *
 * Plain pointers and sizes only.  All device pointers are CUDA global memory
 * of the current device; `stream` is a cudaStream_t (NULL = legacy default
 * stream).  Every call is asynchronous and stream-ordered, allocates no
 * memory (nkimoe_moe_block_host creates two copy streams and a few events per
 * device, and per workspace, when first used), and returns NKIMOE_OK or an
 * error code; nkimoe_last_error() gives the
 * calling thread's last message.  Device-side faults that cannot be detected
 * at launch (an expert id out of range, a bounded wait that ran out) are
 * accumulated in a status word at the start of the caller's workspace and
 * read with nkimoe_read_status().
 *
 * Reference interfaces (Goomelo/nki-moe, Python/NKI) replaced by each entry
 * point are cited as file:line.
 */
#ifndef NKIMOE_H_
#define NKIMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NKIMOE_API __attribute__((visibility("default")))
#else
#define NKIMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define NKIMOE_OK 0
#define NKIMOE_ERR_INVALID_ARG 1   /* bad pointer, shape, dtype or alignment   */
#define NKIMOE_ERR_UNSUPPORTED 2   /* shape outside what the kernels handle    */
#define NKIMOE_ERR_WORKSPACE 3     /* workspace too small                      */
#define NKIMOE_ERR_CUDA 4          /* a CUDA runtime/driver call failed        */
#define NKIMOE_ERR_DEVICE 5        /* nkimoe_read_status: device flagged a fault */

/* device status bits (nkimoe_read_status) */
#define NKIMOE_DEV_TIMEOUT 1       /* a bounded device-side wait ran out       */
#define NKIMOE_DEV_BAD_INDEX 2     /* an expert id outside [0, num_experts) or a cache position outside [0, max_seq) */

/* dtype codes */
#define NKIMOE_F32 0
#define NKIMOE_BF16 1
#define NKIMOE_I32 2
#define NKIMOE_I64 3

/* weight layouts accepted by the packing entry points */
#define NKIMOE_LAYOUT_NXD 0        /* gate_up [E,H,2I], down [E,I,H] (qwen.py:164-226)          */
#define NKIMOE_LAYOUT_HF 1         /* gate_up [E,2I,H], down [E,H,I] (HF Qwen3MoeExperts)       */

#define NKIMOE_IPC_HANDLE_BYTES 64 /* cudaIpcMemHandle_t, for nkimoe_peer_alloc / nkimoe_peer_open */
#define NKIMOE_NOALLOC_SCRATCH_BYTES (8u << 20) /* scratch array of nkimoe_moe_block_noalloc */

NKIMOE_API int nkimoe_version(void);
NKIMOE_API const char* nkimoe_last_error(void);
/* Process-wide tuning knobs: "gemm_schedule" (0 auto, 1 rows on one SM,
 * 2 weights, 3 rows on an SM pair, 4 features x rows on an SM pair, 5 rows
 * on an SM pair over each expert's whole 256-row blocks and on one SM past
 * them),
 * "weights_rows" (16, 32 or 64 rows per decode tile), "weights_balance"
 * (1, the default: a decode GEMM deals its tiles evenly to as many CTAs as
 * its waves need, so the weight stream does not end with a few CTAs reading
 * alone; 0: every CTA strides over the tiles), "router" (0 auto,
 * 1 CUDA-core fp32, 2 tensor-core split-fp32), "prefetch" (64-wide K blocks
 * of a prefill GEMM CTA's next tile pulled into L2 when it starts a tile;
 * 0 = off),
 * "gather_fused" (GEMM-1 loads its token rows itself instead of a separate
 * gather kernel writing them out: 1 with cp.async in its producer warp,
 * 2 with TMA tile::gather4; 0 = separate gather kernel),
 * "epilogue_staging" (prefill GEMM bf16 outputs written through a per-warp
 * shared-memory tile as whole-sector row stores: bit 0 the SwiGLU output,
 * bit 1 the routing-weight-scaled output; default 3),
 * "router_permutes" (1, the default: a decode router of 9 to 255 tokens
 * also writes the expert permutation in its last CTA; 0: a separate
 * permutation launch),
 * "router_halves" (1, the default: the tensor-core router runs two CTAs per
 * 128-row block, one per half of the experts; 0: one CTA over all 128),
 * "router_fused" (1, the default: the tensor-core router forms the summed
 * fp32 logits of its three weight planes in one kernel before the top-k;
 * 0: the grouped GEMM writes the three planes' partials, which the top-k
 * kernel adds),
 * "pdl" (1, the default: the decode-path kernels are launched with
 * programmatic dependent launch, so a kernel's launch and prologue overlap
 * the previous kernel in the stream; 0 = plain launches),
 * "peer_wait_cycles" (budget of each expert-parallel wait for the peers, in
 * SM clock cycles, 1000 to 1e12; default 2e10, about 10 s),
 * "ep_overlap" (schedule of nkimoe_ep_peer_forward: 0 one expert block after
 * every row has arrived; 1 sends, computes and returns overlapped, the send
 * and return kernels storing over NVLink from a side stream; 2 the same with
 * the rows and sums gathered into local staging and moved by the copy
 * engines; -1, the default, picks 2 on 2 to 4 ranks when max_tokens >= 1024
 * and 0 otherwise),
 * "ep_groups" (remote regions taken in this many groups by the overlapped
 * schedules, 1 to 7; 0 = auto, min(ranks - 1, 2)),
 * "ep_side_ctas" (grid bound of the send and return kernels that run beside
 * the expert GEMMs; 0 = the SM count).
 * No reference counterpart (NKI tile sizes are compile-time constants,
 * nki_moe_expert.py:545-556).  Returns NKIMOE_OK or
 * NKIMOE_ERR_INVALID_ARG for an unknown name/value. */
NKIMOE_API int nkimoe_set_option(const char* name, long long value);

/* Profiling hook: `events` is an array of `count` (<= 13) cudaEvent_t that
 * the calling thread's later block calls record on their stream at the start
 * of each stage: 0 router, 1 top-k, 2 permute, 3 gather, 4 GEMM-1 (SwiGLU),
 * 5 GEMM-2 (routing weight), 6 combine, 7 end.  The expert-parallel block
 * (nkimoe_ep_peer_forward) records 0 and 1, then 2 at the (token, rank)
 * sort and 8 once the sends are issued; one-block schedule ("ep_overlap" 0):
 * 9 wait for the senders, 2-7 of the receiver's block (7 after the return
 * of its sums), 10 wait for the partial sums, 11 their sum, 12 end;
 * overlapped schedule: 9 after the own tokens' first half of the experts,
 * 10 after the remote groups, 11 after the second half, the returns and the
 * wait for the partial sums, 12 end.  count = 0 turns it off.
 * No reference counterpart (the reference times whole graphs, main.py:258-277). */
NKIMOE_API int nkimoe_set_stage_events(void* const* events, int count);

/* ---------------------------------------------------------------- norms */

/* nki_rmsnorm_kernel(input_tensor[N,H], weight[H], eps) -> [N,H]
 * (nki_custom_rmsnorm.py:8-70; module NKIRMSNorm.forward :96-123).
 * x_dtype/out_dtype: F32 or BF16; w_dtype: F32 or BF16.  H % 8 == 0. */
NKIMOE_API int nkimoe_rmsnorm(const void* x, int x_dtype, const void* weight, int w_dtype, void* out, int out_dtype,
                   int64_t rows, int64_t hidden, float eps, void* stream);

/* residual_out = x + residual (bf16); out = rmsnorm(residual_out) (bf16).
 * The decoder's residual add feeding post_attention_layernorm
 * (qwen_with_nki.py:447-452).  residual_out may alias residual or x. */
NKIMOE_API int nkimoe_add_rmsnorm(const void* x, const void* residual, void* residual_out, const void* weight, int w_dtype,
                       void* out, int64_t rows, int64_t hidden, float eps, void* stream);

/* Per-head q/k RMSNorm then rotate-half RoPE on a fused bf16 QKV row
 * [T, (n_heads + 2*n_kv_heads) * head_dim] laid out [Q | K | V]
 * (q_layernorm/k_layernorm qwen_with_nki.py:349-350, RotaryEmbedding
 * :330-334; NKI counterpart nki_rope_kernel nki_attention.py:172-249, whose
 * interleaved-pair convention is NOT followed).  positions: int64 [T].
 * qkv_out may equal qkv_in.  head_dim must be 128. */
NKIMOE_API int nkimoe_qk_norm_rope(const void* qkv_in, void* qkv_out, const void* q_weight, const void* k_weight, int w_dtype,
                        const int64_t* positions, int64_t tokens, int n_heads, int n_kv_heads, int head_dim,
                        float rope_theta, float eps, void* stream);

/* ---------------------------------------------------------------- decode attention */

/* Workspace of nkimoe_decode_attention: a status word, one counter per
 * (sequence, kv head) and the split partials.  It must be zero-filled once
 * before its first use; every call leaves the counters at zero again. */
NKIMOE_API size_t nkimoe_decode_attention_workspace_bytes(int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                                          int64_t max_seq);

/* One decode step of grouped-query attention over a KV cache, fused with its
 * inputs' preparation: for every sequence b at position p = positions[b *
 * pos_stride] (pos_stride 0: one position for all), the step's fused QKV row
 * qkv [B, (n_heads + 2*n_kv_heads) * 128] (bf16, before the q/k norms) gets
 * per-head q/k RMSNorm + rotate-half RoPE (as nkimoe_qk_norm_rope), the new
 * key and value are stored at position p of k_cache/v_cache
 * [B, n_kv_heads, max_seq, 128] (bf16, one layer), and query head h attends,
 * with weight softmax(scale * q.k), to positions 0..p of kv head
 * h / (n_heads / n_kv_heads).  out: bf16 [B, n_heads * 128], the layout the
 * O projection takes.  Positions outside [0, max_seq) are reported through
 * the status word (NKIMOE_DEV_BAD_INDEX) and their rows are left unwritten.
 * Reference: nki_flash_attention_decode (nki_attention.py:252-373, online
 * softmax :333-359) with the q/k norms and RoPE of qwen_with_nki.py:330-350;
 * the reference's kernel takes pre-rotated q/k and keeps no cache. */
NKIMOE_API int nkimoe_decode_attention(const void* qkv, const void* q_weight, const void* k_weight, int w_dtype,
                                       const int64_t* positions, int64_t pos_stride, void* k_cache, void* v_cache,
                                       void* out, int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                       int64_t max_seq, float rope_theta, float eps, float scale, void* workspace,
                                       size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- decode projections */

/* y[M, N] = x[M, K] . w[N, K]^T for decode batches, M <= 16 (bf16 in and out,
 * fp32 accumulation, deterministic); w in the nn.Linear layout [out, in].
 * N % 16 == 0, K % 32 == 0, pointers 16-byte aligned.  Streams w once at
 * HBM rate.  The decode step's projections: nki_qkv_projection
 * (nki_attention.py:32-169), the O projection (qwen_with_nki.py:330-350) and
 * the LM head (qwen_with_nki.py:495); NKI tile matmul nki_matmul_tiled
 * (nki_moe_integrated.py:27-84). */
NKIMOE_API int nkimoe_skinny_linear(const void* x, const void* w, void* y, int64_t M, int64_t N, int64_t K,
                                    void* stream);

/* ---------------------------------------------------------------- router */

/* logits[T,E] (fp32) = x(bf16)[T,H] . router_w(fp32)[E,H]^T (+ router_bias[E])
 * (NKIMoESimple.router, nki_moe_integrated.py:411-412, :437). */
NKIMOE_API int nkimoe_router_logits(const void* x, const float* router_w, const float* router_bias, float* logits, int64_t T,
                         int64_t H, int64_t E, void* stream);

/* Splits fp32 router weights [E,H] into three bf16 planes [3, E, H] =
 * (hi, mid, lo) with hi + mid + lo == w exactly, for the tensor-core router
 * of nkimoe_moe_block: with bf16 activations every product is exact and the
 * accumulation is fp32, so the logits are fp32 logits.  No reference
 * counterpart (the reference computes the fp32 router with nn.Linear,
 * nki_moe_integrated.py:437). */
NKIMOE_API int nkimoe_router_split(const float* router_w, void* router_w_split, int64_t E, int64_t H, void* stream);

/* softmax -> top-k (descending; ties to the lower expert id) -> renormalise
 * (nki_moe_integrated.py:438-443).  idx int32 [T,K], w fp32 [T,K]. */
NKIMOE_API int nkimoe_topk_softmax(const float* logits, int64_t T, int64_t E, int64_t K, int32_t* topk_idx, float* topk_w,
                        void* stream);

/* ---------------------------------------------------------------- permutation */

NKIMOE_API size_t nkimoe_permute_workspace_bytes(int64_t T, int64_t K, int64_t E);

/* Stable grouping of the T*K assignments by expert, (k, t) order inside an
 * expert (nki_moe_integrated.py:450-467).  topk_idx is [T,K] of idx_dtype
 * (I32 or I64); a negative id is an empty slot, an id >= E an error.  Outputs:
 * row_token[T*K], row_slot[T*K] (= t*K + k), slot_row[T*K] (inverse; -1 for
 * an empty or out-of-range slot), expert_offsets[E+1]. */
NKIMOE_API int nkimoe_permute(const void* topk_idx, int idx_dtype, int64_t T, int64_t K, int64_t E, int32_t* row_token,
                   int32_t* row_slot, int32_t* slot_row, int32_t* expert_offsets, void* workspace,
                   size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- weights */

/* Packs gate_up_proj into the GEMM layout W13 [E, 2I, H] bf16: K-major, row
 * blocks of 128 = [gate 64 | up 64].  layout: NKIMOE_LAYOUT_NXD for the
 * reference's [E,H,2I] (qwen.py:164-202), NKIMOE_LAYOUT_HF for [E,2I,H].
 * I % 64 == 0, H % 64 == 0. */
NKIMOE_API int nkimoe_pack_gate_up(const void* gate_up, int layout, void* w13, int64_t E, int64_t H, int64_t I, void* stream);

/* Packs down_proj into W2 [E, H, I] bf16 (K-major).  layout NXD: [E,I,H]
 * (qwen.py:204-226) is transposed; HF: [E,H,I] is copied. */
NKIMOE_API int nkimoe_pack_down(const void* down, int layout, void* w2, int64_t E, int64_t H, int64_t I, void* stream);

/* ---------------------------------------------------------------- MoE block */

NKIMOE_API size_t nkimoe_moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K);

/* Expert stage given routing: out[T,H] (bf16) = sum_k w[t,k] *
 * FFN_{idx[t,k]}(x[t]); a negative idx[t,k] marks an empty slot.  The whole-block kernels nki_moe_full_forward /
 * nki_moe_optimized (nki_moe_kernel.py:185-423), nki_moe_expert_kernel /
 * nki_moe_expert_fused_kernel_v2 (nki_moe_expert.py:21-355), all
 * (hidden_states[T,H], gate_up_proj, down_proj, expert_indices[T,K],
 * expert_weights[T,K]) -> [T,H].  x bf16 [T,H]; w13/w2 packed (above);
 * topk_idx [T,K] of idx_dtype; topk_w fp32 [T,K]. */
NKIMOE_API int nkimoe_moe_experts(const void* x, const void* w13, const void* w2, const void* topk_idx, int idx_dtype,
                       const float* topk_w, void* out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Whole block, router included: NKIMoESimple.forward
 * (nki_moe_integrated.py:428-475) and NKIMoEWrapper._nki_forward (:292-387).
 * router_w fp32 [E,H]; router_bias fp32 [E] or NULL; router_w_split (from
 * nkimoe_router_split) or NULL: when given, large token counts run the router
 * on the tensor cores; topk_idx_out (int32 [T,K]) and topk_w_out (fp32 [T,K])
 * may be NULL. */
NKIMOE_API int nkimoe_moe_block(const void* x, const float* router_w, const float* router_bias,
                     const void* router_w_split, const void* w13, const void* w2,
                     void* out, int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E,
                     int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* nkimoe_moe_block followed by the decoder's residual add and the next
 * RMSNorm (qwen_with_nki.py:447-454 with NKIRMSNorm, nki_custom_rmsnorm.py):
 * residual_out = residual + block(x) (bf16) and norm_out =
 * rmsnorm(residual_out) * norm_w (bf16), all [T, H]; residual_out may alias
 * residual; norm_w_dtype F32 or BF16.  Same workspace as nkimoe_moe_block.
 * Up to 512 tokens the block's combine and the norm run as one kernel; the
 * results equal nkimoe_moe_block + nkimoe_add_rmsnorm bit for bit. */
NKIMOE_API int nkimoe_moe_block_add_rmsnorm(const void* x, const float* router_w, const float* router_bias,
                                            const void* router_w_split, const void* w13, const void* w2,
                                            const void* residual, void* residual_out, const void* norm_w,
                                            int norm_w_dtype, float eps, void* norm_out, int32_t* topk_idx_out,
                                            float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                                            void* workspace, size_t workspace_bytes, void* stream);

/* The block with the post-attention RMSNorm inside it: x = rmsnorm(h) *
 * norm_w (bf16, as nkimoe_rmsnorm), then nkimoe_moe_block on x.  This is the
 * reference's fused-norm MoE (qwen_with_nki.py:379-382 passes
 * post_attention_layernorm into the MoE module when moe_fused_nki_kernel_enabled,
 * and :451-452 then skips the decoder's own norm call).  For prefill batches
 * (more than 512 tokens, router_w_split given, 128 experts) the norm and the
 * router logits run as one tensor-core kernel that writes the normalised rows
 * once and routes them in the same pass (the top-k kernel follows); smaller
 * batches run the RMSNorm kernel and then the router.  Either way the results equal
 * nkimoe_rmsnorm + nkimoe_moe_block bit for bit.  x_out [T, H] bf16 (device,
 * may be NULL: the rows then stay in the workspace); norm_w_dtype F32 or
 * BF16; workspace nkimoe_moe_block_rmsnorm_workspace_bytes. */
NKIMOE_API size_t nkimoe_moe_block_rmsnorm_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K);
NKIMOE_API int nkimoe_moe_block_rmsnorm(const void* h, const void* norm_w, int norm_w_dtype, float eps, void* x_out,
                                        const float* router_w, const float* router_bias, const void* router_w_split,
                                        const void* w13, const void* w2, void* out, int32_t* topk_idx_out,
                                        float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                                        void* workspace, size_t workspace_bytes, void* stream);

/* Whole block on HOST buffers: NKIMoESimple called on a host tensor
 * (test_nki_moe.py:146-151 runs the module on hidden_states created on the
 * host; nki_moe_integrated.py:428-475 is its forward).  x_host [T,H] bf16 in,
 * out_host [T,H] bf16 out, both page-locked for the copies to overlap
 * (pageable buffers work, with the copies synchronous); the weights, the
 * routing outputs (device pointers, may be NULL) and the workspace
 * (nkimoe_moe_block_host_workspace_bytes) are on the current device.
 * The copies run on two streams of the library (one per direction and
 * device), ordered against `stream` by events:
 *  - within a call, the tokens go through in chunks: the copy of chunk c+1
 *    to the device and of chunk c-1 to the host overlap the block on chunk c.
 *    chunk_tokens <= 0 picks half the batch; chunk_tokens >= T, one chunk.
 *    Chunks are cut only where each takes the whole batch's router and GEMM
 *    paths (router_w_split given, 256 tokens or more, more than 48 rows per
 *    expert under the auto schedule), so out equals nkimoe_moe_block's on the
 *    whole batch bit for bit; otherwise one chunk;
 *  - across calls, the workspace holds two slots of staging rows used by
 *    alternate calls: a call's copy to the device overlaps the previous
 *    call's block, and with done_event its copy back overlaps the next call's
 *    block.
 * done_event NULL: `stream` completes with the last copy to the host.
 * done_event (a cudaEvent_t of this device): recorded at the last copy to the
 * host, which `stream` does not wait for; out_host is ready once the event
 * has completed.  The host buffers must stay valid until then, and no other
 * entry point may be given the workspace before then (the copy back reads
 * the call's staging rows in it); host-batch calls that share a workspace
 * are issued on one stream and alternate its two slots safely.  The slots'
 * place in the workspace follows T: a call whose T differs from the previous
 * call's on the same workspace first waits for the earlier calls' blocks and
 * copies back (no overlap across that change).  Returns once
 * the work is enqueued.  The status word of the workspace
 * (nkimoe_read_status) collects the call's device faults. */
NKIMOE_API size_t nkimoe_moe_block_host_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K);
/* How nkimoe_moe_block_host cuts a T-token batch under the current options:
 * chunks of *chunk_len tokens, *chunk_count of them, the last taking the
 * remainder (T - (count - 1) * len).  Host-only; no reference counterpart. */
NKIMOE_API int nkimoe_moe_block_host_plan(int64_t T, int64_t E, int64_t K, int have_router_split,
                                          int64_t chunk_tokens, int64_t* chunk_len, int64_t* chunk_count);
NKIMOE_API int nkimoe_moe_block_host(const void* x_host, const float* router_w, const float* router_bias,
                                     const void* router_w_split, const void* w13, const void* w2, void* out_host,
                                     int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I,
                                     int64_t E, int64_t K, int64_t chunk_tokens, void* workspace,
                                     size_t workspace_bytes, void* done_event, void* stream);

/* nkimoe_moe_block for callers that cannot allocate GPU memory (a server that
 * reserved all device memory up front, a runtime whose allocator may not be
 * entered where the layer is issued, an embedding that forbids allocation
 * while it records CUDA graphs).  It has no counterpart in the reference.
 * Same arguments and results as nkimoe_moe_block without the workspace: the
 * scratch is a fixed NKIMOE_NOALLOC_SCRATCH_BYTES (8 MiB) array inside the
 * library, held by every GPU that loads the library until the process exits.
 * A batch fits when nkimoe_moe_workspace_bytes(T, H, I, E, K) is at most that
 * size: up to 175 tokens at H=2048, I=768, E=128, K=8.  Larger batches return
 * NKIMOE_ERR_WORKSPACE, and bad shapes NKIMOE_ERR_INVALID_ARG or
 * NKIMOE_ERR_UNSUPPORTED, without touching the GPU.  Device faults (a bounded
 * wait that ran out, an expert id out of range) land in the array's status
 * word: read it with nkimoe_noalloc_read_status.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) and should come before any
 * stream capture.  All calls on a device share the array, which keeps the
 * last call's contents (each call clears what must start at zero): two calls
 * that overlap on the GPU, e.g. issued on two streams or from two host
 * threads without ordering, race on it. */
NKIMOE_API int nkimoe_moe_block_noalloc(const void* x, const float* router_w, const float* router_bias,
                                        const void* router_w_split, const void* w13, const void* w2, void* out,
                                        int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I,
                                        int64_t E, int64_t K, void* stream);
/* Reads and clears the status word of nkimoe_moe_block_noalloc's scratch
 * array on the current device (synchronises the stream; allocates nothing).
 * Same returns as nkimoe_read_status.  No reference counterpart. */
NKIMOE_API int nkimoe_noalloc_read_status(void* stream, int* status_out);

/* Reads and clears the device status word of a workspace (synchronises the
 * stream).  Returns NKIMOE_OK, NKIMOE_ERR_DEVICE (status in *status_out), or
 * NKIMOE_ERR_CUDA. */
NKIMOE_API int nkimoe_read_status(void* workspace, void* stream, int* status_out);

/* ---------------------------------------------------------------- expert parallel */
/* The expert-parallel block splits nkimoe_moe_block into the pieces around
 * its two all-to-all exchanges (NCCL, issued by the host layer).  The
 * reference has no kernels for them: its EP lives inside NxDI
 * (moe_ep_degree, qwen.py:272, :515). */

NKIMOE_API size_t nkimoe_route_workspace_bytes(int64_t T, int64_t H, int64_t E, int64_t K);

/* Router + softmax/top-k/renormalise only (nki_moe_integrated.py:436-443):
 * int32 topk_idx [T,K], fp32 topk_w [T,K]. */
NKIMOE_API int nkimoe_route(const void* x, const float* router_w, const float* router_bias, const void* router_w_split,
                            int32_t* topk_idx, float* topk_w, int64_t T, int64_t H, int64_t E, int64_t K,
                            void* workspace, size_t workspace_bytes, void* stream);

NKIMOE_API size_t nkimoe_dispatch_workspace_bytes(int64_t T, int64_t K, int64_t E);

/* Permutation by global expert and row gather: x_perm [T*K, H] bf16 in
 * (expert, k, t) order, so the rows for the ranks owning experts
 * [r*E/P, (r+1)*E/P) are contiguous; row_weight [T*K] the routing weight of
 * each permuted row; slot_row [T*K] the inverse permutation (for
 * nkimoe_combine); expert_counts [E] rows per expert.  Follows the dispatch
 * order of nki_moe_integrated.py:450-467. */
NKIMOE_API int nkimoe_dispatch(const void* x, const void* topk_idx, int idx_dtype, const float* topk_w, int64_t T,
                               int64_t H, int64_t E, int64_t K, void* x_perm, float* row_weight, int32_t* slot_row,
                               int32_t* expert_counts, void* workspace, size_t workspace_bytes, void* stream);

NKIMOE_API size_t nkimoe_segment_experts_workspace_bytes(int64_t rows, int64_t I, int64_t segments);

/* Expert FFNs over `segments` consecutive row segments of a (bf16 [rows, H]);
 * segment s has segment_counts[s] rows (device int32) and uses local expert
 * s % experts_per_group of w13 [experts_per_group, 2I, H] / w2 [.., H, I];
 * y [rows, H] bf16 = row_weight[r] * FFN(a[r]).  With segments ordered
 * (source rank, local expert) this runs on the rows an all-to-all delivered
 * without re-sorting them (nki_moe_integrated.py:142-206 per expert). */
NKIMOE_API int nkimoe_segment_experts(const void* a, const float* row_weight, const int32_t* segment_counts,
                                      int64_t segments, int64_t experts_per_group, const void* w13, const void* w2,
                                      void* y, int64_t rows, int64_t H, int64_t I, void* workspace,
                                      size_t workspace_bytes, void* stream);

NKIMOE_API size_t nkimoe_ep_dispatch_workspace_bytes(int64_t T, int64_t P);

/* De-duplicated expert-parallel dispatch over P ranks with experts_per_rank
 * experts each (rank d owns [d*El, (d+1)*El)): one send row per (token, rank)
 * pair that has at least one of the token's experts, rows grouped by rank and
 * ordered by token.  Outputs x_send [<= T*P, H] bf16, slots_send [.., K] int32
 * (the token's K slots as the destination sees them: local expert id or -1),
 * weights_send [.., K] fp32 (routing weight, 0 for -1 slots), rank_counts [P]
 * rows per rank, slot_row [T, P] (row of (t, d) or -1) for the final
 * nkimoe_combine with K = P.  The receiver runs nkimoe_moe_experts on the
 * rows with slots/weights as routing (negative ids are empty slots). */
NKIMOE_API int nkimoe_ep_dispatch(const void* x, const int32_t* topk_idx, const float* topk_w, int64_t T, int64_t H,
                                  int64_t K, int64_t num_ranks, int64_t experts_per_rank, void* x_send,
                                  int32_t* slots_send, float* weights_send, int32_t* rank_counts, int32_t* slot_row,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* out[t] = sum_k (slot_weight ? slot_weight[t*K+k] : 1) * y[slot_row[t*K+k]]
 * in fp32, k ascending, bf16 out (nki_moe_integrated.py:482-494,
 * nki_moe_aggregate :209-251); slot_row < 0 is skipped.  T * H / 8 and
 * T * K below 2^31 (NKIMOE_ERR_UNSUPPORTED otherwise). */
NKIMOE_API int nkimoe_combine(const void* y, const int32_t* slot_row, const float* slot_weight, void* out, int64_t T,
                              int64_t K, int64_t H, void* stream);

/* ---------------------------------------------------------------- expert parallel over peer memory
 *
 * No reference counterpart: the reference's expert parallelism is NxDI's
 * (qwen.py:35, :240), which is not in the reference tree.  This is the
 * one-process-per-GPU exchange of this library: every rank allocates one
 * exchange buffer (nkimoe_peer_alloc), the ranks swap the IPC handles (through
 * their process group), and each opens the others' buffers (nkimoe_peer_open).
 * No multicast object is created; peers are reached by plain NVLink stores. */

/* Bytes of one rank's exchange buffer for num_ranks ranks of at most
 * max_tokens tokens each. */
NKIMOE_API size_t nkimoe_ep_peer_buffer_bytes(int64_t num_ranks, int64_t max_tokens, int64_t H, int64_t K);

/* cudaMalloc (zero-filled) + its IPC handle (NKIMOE_IPC_HANDLE_BYTES bytes). */
NKIMOE_API int nkimoe_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another process's buffer (cudaIpcOpenMemHandle, peer access enabled). */
NKIMOE_API int nkimoe_peer_open(const void* ipc_handle, void** ptr);
NKIMOE_API int nkimoe_peer_close(void* ptr);
NKIMOE_API int nkimoe_peer_free(void* ptr);

NKIMOE_API size_t nkimoe_ep_peer_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                                                 int64_t num_ranks, int64_t max_tokens);

/* The schedule nkimoe_ep_peer_forward takes for num_ranks ranks and buffers of
 * max_tokens rows under the current "ep_overlap" option: 0 one block, 1
 * overlapped with SM stores, 2 overlapped with copy engines.  Host-only; no
 * reference counterpart. */
NKIMOE_API int nkimoe_ep_peer_schedule(int64_t num_ranks, int64_t max_tokens);

/* The expert-parallel MoE block for this rank's T <= max_tokens tokens, one
 * stream-ordered call with no host synchronisation: route (as
 * nkimoe_moe_block) -> each token's row sent once to every rank owning one of
 * its experts (stores into that rank's buffer) -> wait for the num_ranks
 * senders -> this rank's experts (w13_local/w2_local: packed weights of
 * experts [rank*E/P, (rank+1)*E/P)) over the received rows -> each row's
 * weighted sum stored back into its source's buffer -> wait -> sum of the
 * num_ranks partial sums into out [T, H].  peer_buffers: the num_ranks
 * buffers as mapped in this process (this rank's own at index rank).  Every
 * rank calls this once per step with the same epoch, increasing between
 * steps; epoch 0 lets each rank's buffer count the steps on the device (its
 * own counter + 1 per call), so that a step captured in a CUDA graph can be
 * replayed -- a caller uses one mode for the buffer's lifetime.  The default
 * overlapped schedule (option "ep_overlap") issues the sends, one
 * destination after another nearest first, on a side stream of the library
 * while this rank's experts run over its own tokens; it takes the remote rows
 * in groups as they arrive and returns each group's sums from the side
 * stream while the next group computes; the call's work on the side stream
 * is joined back into `stream` before the final sum (capturable; the first
 * call on a device creates the side stream and should come before any
 * capture).  Calls on one device share the side stream.  A peer that
 * never arrives sets NKIMOE_DEV_TIMEOUT in the status word
 * (nkimoe_read_status) after a bounded wait (~10 s; option
 * "peer_wait_cycles").  topk_idx_out / topk_w_out (device, [T, K], may be
 * NULL): the routing of this rank's tokens, as nkimoe_moe_block returns it. */
NKIMOE_API int nkimoe_ep_peer_forward(const void* x, const float* router_w, const float* router_bias,
                                      const void* router_w_split, const void* w13_local, const void* w2_local,
                                      void* out, int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H,
                                      int64_t I, int64_t E, int64_t K,
                                      int64_t num_ranks, int64_t rank, int64_t max_tokens, void* const* peer_buffers,
                                      uint32_t epoch, void* workspace, size_t workspace_bytes, void* stream);

/* nkimoe_ep_peer_forward with hot-expert replicas: every rank holds
 * local_slots expert slots (its own experts and copies of other ranks' hot
 * experts; slot v is local expert v % local_slots of rank v / local_slots;
 * w13_local / w2_local hold this rank's local_slots packed experts).
 * expert_slots (device int32 [E, max_holders]) lists, for expert e, the
 * slot_counts[e] (device int32 [E], 1..max_holders) slots that hold its
 * weights; slot k of token t with expert e goes to slot expert_slots[e *
 * max_holders + t mod slot_counts[e]], so an expert's tokens are split evenly
 * over its holders.  With every slot_counts[e] = 1 and expert e at slot e
 * (local_slots = E / P) this is nkimoe_ep_peer_forward.  Every rank passes
 * the same tables.  The partial sums a token gets back come from the ranks
 * its slots went to, so the output meets the block tolerance against the
 * single-GPU block (as without replicas); the returned routing is the real
 * expert ids.  An entry outside [0, num_ranks * local_slots) drops its slot
 * and sets NKIMOE_DEV_BAD_INDEX.  The reference has no counterpart (NxDI's
 * moe_ep_degree partitions experts statically, qwen.py:272, :515). */
NKIMOE_API size_t nkimoe_ep_peer_workspace_bytes_mapped(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                                                        int64_t num_ranks, int64_t max_tokens, int64_t local_slots);
NKIMOE_API int nkimoe_ep_peer_forward_mapped(const void* x, const float* router_w, const float* router_bias,
                                             const void* router_w_split, const void* w13_local,
                                             const void* w2_local, void* out, int32_t* topk_idx_out,
                                             float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E,
                                             int64_t K, int64_t num_ranks, int64_t rank, int64_t max_tokens,
                                             void* const* peer_buffers, uint32_t epoch, void* workspace,
                                             size_t workspace_bytes, void* stream, int64_t local_slots,
                                             const int32_t* expert_slots, const int32_t* slot_counts,
                                             int64_t max_holders);

/* ---------------------------------------------------------------- pieces */

/* Grouped GEMM over expert segments: for each expert e, rows
 * [offsets[e], offsets[e+1]) of a (bf16 [M, Kd], K-major) times w_packed[e]
 * (bf16 [N, Kd], K-major); out bf16 [M, N] (or [out_rows, N] through
 * out_row_map).  nki_grouped_expert_gemm(input_tokens[M,H],
 * expert_weights[E,H,N], expert_ids[M], num_experts) (nki_moe_expert.py:466-542)
 * and nki_matmul_tiled(a[M,K], b[K,N]) (nki_moe_integrated.py:27-84, E = 1).
 * expert_offsets is a device int32 [E+1]; status: device int or NULL. */
NKIMOE_API int nkimoe_grouped_gemm(const void* a, const void* w_packed, const int32_t* expert_offsets, const int32_t* out_row_map,
                        void* out, int64_t M, int64_t N, int64_t Kd, int64_t E, int* status, void* stream);

/* silu(gate) * up over a bf16 [M, 2N] gate|up split (nki_swiglu,
 * nki_moe_integrated.py:87-139). */
NKIMOE_API int nkimoe_swiglu(const void* gate_up, void* out, int64_t M, int64_t N, void* stream);

/* Sum over the leading top-k axis of bf16 [K, T, H] (nki_moe_aggregate,
 * nki_moe_integrated.py:209-251). */
NKIMOE_API int nkimoe_aggregate(const void* expert_outputs, void* out, int64_t K, int64_t T, int64_t H, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NKIMOE_H_ */
