// Internal launch interface between the C-ABI layer (capi.cu) and the kernel
// translation units.  Everything here is stream-ordered and allocation-free.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace nkimoe {

// dtype codes shared with include/nkimoe.h
constexpr int kF32 = 0;
constexpr int kBF16 = 1;
constexpr int kI32 = 2;
constexpr int kI64 = 3;

constexpr int kMaxExperts = 512;

// Launch with programmatic dependent launch (see pdl_wait in common.cuh) when
// the "pdl" option is on (the default); the kernel must call pdl_wait()
// before touching global memory.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Stages of a block call, in launch order (for nkimoe_set_stage_events).
enum Stage : int {
  kStageRouter = 0,
  kStageTopk = 1,
  kStagePermute = 2,
  kStageGather = 3,
  kStageGemm1 = 4,
  kStageGemm2 = 5,
  kStageCombine = 6,
  kStageEnd = 7,
  // expert-parallel block only: the exchange around the receiver's block
  kStageEpSend = 8,        // destinations, (token, rank) sort and the rows' stores to their owners
  kStageEpWait = 9,        // wait for the senders, mask of unused region rows
  kStageEpReturnWait = 10, // after the receiver's block: wait for the partial sums
  kStageEpSum = 11,        // sum of the partial sums
  kStageEpEnd = 12,
  kNumStageEvents = 13,
};
constexpr int kPermuteChunk = 256;  // assignments per block in the permutation kernels

// ----------------------------------------------------------------- norms
cudaError_t rmsnorm_launch(const void* x, int x_dtype, const void* w, int w_dtype, void* out, int out_dtype,
                           long long rows, int hidden, float eps, cudaStream_t s);
cudaError_t add_rmsnorm_launch(const void* x, const void* residual, void* residual_out, const void* w, int w_dtype,
                               void* out, long long rows, int hidden, float eps, cudaStream_t s);
// The MoE block's combine (rows of y already scaled by their routing weight)
// fused with the next residual add + RMSNorm, rows <= 512 (one CTA per row).
bool combine_add_rmsnorm_supported(long long rows, int hidden);
cudaError_t combine_add_rmsnorm_launch(const __nv_bfloat16* y, const int32_t* slot_row, int K,
                                       const __nv_bfloat16* residual, __nv_bfloat16* residual_out, const void* w,
                                       int w_dtype, __nv_bfloat16* out, long long rows, int hidden, float eps,
                                       cudaStream_t s);
cudaError_t qk_norm_rope_launch(const void* qkv_in, void* qkv_out, const void* qw, const void* kw, int w_dtype,
                                const long long* positions, long long tokens, int n_heads, int n_kv, int head_dim,
                                float theta, float eps, cudaStream_t s);

// ----------------------------------------------------------------- decode attention
int decode_attention_chunk(int max_seq);
size_t decode_attention_workspace_bytes(long long B, int n_heads, int n_kv, int max_seq);
cudaError_t decode_attention_launch(const __nv_bfloat16* qkv, const void* qw, const void* kw, int w_dtype,
                                    const long long* positions, long long pos_stride, __nv_bfloat16* k_cache,
                                    __nv_bfloat16* v_cache, __nv_bfloat16* out, int B, int n_heads, int n_kv,
                                    int max_seq, float theta, float eps, float scale, void* workspace,
                                    cudaStream_t s);

// ----------------------------------------------------------------- decode projections
cudaError_t skinny_linear_launch(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int M, int N,
                                 int K, cudaStream_t s);

// ----------------------------------------------------------------- router
// fp32 logits = x(bf16) . Wr(fp32)^T (+ bias), CUDA-core fp32 FMA, fixed order.
cudaError_t router_logits_simt_launch(const __nv_bfloat16* x, const float* wr, const float* bias, float* logits,
                                      int tokens, int hidden, int experts, cudaStream_t s);
// Split fp32 router weights into three bf16 planes [3, E, H] = hi, mid, lo.
cudaError_t router_split_launch(const float* wr, __nv_bfloat16* wsplit, int experts, int hidden, cudaStream_t s);
// Split-K fp32 router for few tokens: partial[split][T][E].
cudaError_t router_splitk_launch(const __nv_bfloat16* x, const float* wr, float* partial, int tokens, int hidden,
                                 int experts, int splits, cudaStream_t s);
int router_splits_for(int tokens, int hidden, int experts);
// softmax -> top-k (by logit, ties to the lower id) -> renormalise.
cudaError_t topk_softmax_launch(const float* logits, int tokens, int experts, int top_k, int32_t* idx, float* w,
                                cudaStream_t s);
// Router logits + softmax + top-k in one launch for few tokens (T < 8 * 48):
// CTAs over (8-expert block, hidden slice, 8-token group) write fp32 partial
// logits [slice][T][E] to `partial`; the last CTA of a token group adds the
// slices in order and selects its top-k.  `counters` (one int per token group,
// zero on entry, left at zero) count the finished CTAs.  Supported when
// E <= 256, H % 128 == 0, 1 <= K <= min(32, E).
bool router_topk_fused_supported(int hidden, int experts, int top_k);
int router_topk_slices(int tokens, int hidden, int experts);
int router_topk_max_groups();
// Outputs of the permutation (permute_launch's) for the decode router to
// fill itself when the batch is one token group (8 tokens or fewer).
struct RouterPermOut {
  int32_t* row_token;
  int32_t* row_slot;
  int32_t* slot_row;
  int32_t* expert_offsets;
  float* row_weight;
  int* status;
};
bool router_topk_fused_permutes(int tokens);
// The same result for more than one token group (measured faster there):
// 8-CTA clusters of 8 tokens, the expert logits of a token gathered over
// distributed shared memory.  Same support conditions; no partials.  With
// `perm` (tokens * top_k <= kPermuteSmall) the last CTA of the grid to finish
// (`counter`: one int, zero on entry, left at zero) also writes the
// permutation, as permute_launch would.
bool router_topk_cluster_permutes(int tokens, int top_k);
cudaError_t router_topk_cluster_launch(const __nv_bfloat16* x, const float* wr, const float* bias, float* logits_out,
                                       int tokens, int hidden, int experts, int top_k, int32_t* idx, float* w,
                                       cudaStream_t s, int* counter = nullptr,
                                       const RouterPermOut* perm = nullptr);
cudaError_t router_topk_fused_launch(const __nv_bfloat16* x, const float* wr, const float* bias, float* logits_out,
                                     int tokens, int hidden, int experts, int top_k, int32_t* idx, float* w,
                                     float* partial, int* counters, cudaStream_t s,
                                     const RouterPermOut* perm = nullptr);
// Same on logits given as `splits` fp32 partial sums [split][T][E] (+ bias[E]);
// logits_out (nullable) receives the summed logits.
// Router logits of a prefill batch on the tensor cores in one kernel (E ==
// 128, the weights as three bf16 planes; tmap_w over [3 E, H], box 64 x
// experts_per_cta (64: two CTAs per 128-row block, one per half of the
// experts; or 128)):
// logits_out [T, E] = ((hi + mid) + lo) + bias, the values topk_softmax
// forms from the router GEMM's three partials, so its top-k is bit for bit the
// two-kernel one.  With h non-null the CTA normalises the rows first (RMSNorm,
// norm_w of dtype F32/BF16, H <= 2048), writes them to x_out and routes them;
// otherwise it routes x through tmap_x (box 64 x 128).
bool router_tc_supported(long long T, int H, int E, bool norm);
cudaError_t router_tc_launch(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const __nv_bfloat16* h,
                             const void* norm_w, int norm_w_dtype, float eps, __nv_bfloat16* x_out, const float* bias,
                             float* logits_out, long long T, int H, int* status, cudaStream_t s,
                             int experts_per_cta);
cudaError_t topk_softmax_partials_launch(const float* partial, int splits, const float* bias, float* logits_out,
                                         int tokens, int experts, int top_k, int32_t* idx, float* w, cudaStream_t s);

// ----------------------------------------------------------------- permutation
size_t permute_scratch_bytes(long long tokens, int top_k, int experts);
cudaError_t permute_launch(const void* idx, int idx_dtype, int tokens, int top_k, int experts, int32_t* row_token,
                           int32_t* row_slot, int32_t* slot_row, int32_t* expert_offsets, void* scratch,
                           int* status, cudaStream_t s, const float* slot_weight = nullptr,
                           float* row_weight = nullptr);
cudaError_t gather_rows_launch(const __nv_bfloat16* x, const int32_t* row_token, const int32_t* expert_offsets,
                               int experts, __nv_bfloat16* x_perm, long long max_rows, int hidden, cudaStream_t s);
cudaError_t combine_launch(const __nv_bfloat16* y, const int32_t* slot_row, const float* slot_weight,
                           __nv_bfloat16* out, int tokens, int top_k, int hidden, cudaStream_t s);
// Expert-parallel de-duplicated dispatch helpers (see permute.cu).
cudaError_t ep_dest_launch(const int32_t* idx, int T, int K, int P, int El, int32_t* dest, cudaStream_t s);
cudaError_t ep_slots_launch(const int32_t* idx, const float* w, const int32_t* row_token, const int32_t* row_slot,
                            const int32_t* rank_offsets, long long max_rows, int P, int K, int El, int32_t* slots,
                            float* wts, cudaStream_t s);
// ----------------------------------------------------------------- expert parallel over peer memory
constexpr int kMaxPeers = 8;
struct EpPeerPtrs {
  char* base[kMaxPeers];  // every rank's exchange buffer, mapped into this process
};
struct EpPeerLayout {  // byte offsets inside an exchange buffer (ep_peer.cu)
  size_t step, disp_flag, res_flag, counts, recv_slots, recv_w, recv_x, ret_y, total;
};
EpPeerLayout ep_peer_layout(long long P, long long max_tokens, long long H, long long K);
// Regions of an exchange buffer are indexed by the distance q = (receiver -
// source) mod P: region q of rank d holds the rows sent by rank d - q, and
// region q of rank s's ret_y the partial sums returned by rank s + q.  Flags
// and counts are indexed the same way.  Region 0 is the rank's own.
//
// Rows (sorted by destination rank: rank_offsets[P + 1]) for the destinations
// d_first .. d_first + d_count - 1 go to region (d - src) mod P of d's
// buffer; the last CTA publishes their counts and raises their dispatch flags.
// max_ctas bounds the grid (0: as many as the rows need).
cudaError_t ep_peer_send_launch(const __nv_bfloat16* x, const int32_t* idx, const float* w, const int32_t* row_token,
                                const int32_t* row_slot, const int32_t* rank_offsets, int T, int H, int K, int P,
                                int El, int Tm, int src, int d_first, int d_count, const EpPeerPtrs& peers,
                                const EpPeerLayout& L, unsigned* counter, const uint32_t* epoch_p, int max_ctas,
                                cudaStream_t s);
// Source-side bookkeeping of a step: the row of every (token t, rank d) partial
// sum in this rank's ret_y (slot_out[t * P + d], -1: no expert of t on d) and,
// when self_idx is given, this rank's own share of its tokens as a given
// routing (self_idx[t][k] = local expert id or -1, self_w the weight or 0);
// with self_direct the own partial sums sit in region 0 at row t, otherwise at
// the row the token was sent to.
cudaError_t ep_peer_local_launch(const int32_t* idx, const float* w, const int32_t* slot_in,
                                 const int32_t* rank_offsets, int T, int K, int P, int El, int Tm, int src,
                                 bool self_direct, int32_t* slot_out, int32_t* self_idx, float* self_w, cudaStream_t s);
// Copy-engine form of the send: the rows of every destination d != src, in
// the order ep_peer_send_launch gives them, written to this rank's staging
// [P][Tm] rows (stage_x, stage_slots, stage_w, stage_counts[d]) instead of
// the peers' buffers; the library then copies each destination's whole
// staging region to it and raises its flag with ep_peer_publish_launch.
cudaError_t ep_peer_stage_launch(const __nv_bfloat16* x, const int32_t* idx, const float* w, const int32_t* row_token,
                                 const int32_t* row_slot, const int32_t* rank_offsets, int T, int H, int K, int P,
                                 int El, int Tm, int src, __nv_bfloat16* stage_x, int32_t* stage_slots,
                                 float* stage_w, int32_t* stage_counts, cudaStream_t s);
// One thread: *count_dst = *count_src (when count_src is given), then, after a
// system-scope fence, *flag = the step's epoch with release semantics.
cudaError_t ep_peer_publish_launch(int32_t* count_dst, const int32_t* count_src, uint32_t* flag,
                                   const uint32_t* epoch_p, cudaStream_t s);
// epoch := value when nonzero, else epoch + 1 (device-side step count)
cudaError_t ep_peer_step_launch(uint32_t* step, uint32_t value, cudaStream_t s);
// Waits (bounded by budget_cycles) until flags[0 .. n) all hold the epoch.
// Hot-expert replicas: idx_v[t, k] = slots[idx[t, k] * max_holders +
// t mod counts[idx[t, k]]], the expert slot (rank * local_slots + local
// expert) that takes slot (t, k); -1 and a status flag for bad entries.
cudaError_t ep_remap_launch(const int32_t* idx, int T, int K, int E, const int32_t* slots, const int32_t* counts,
                            int max_holders, int num_slots, int32_t* idx_v, int* status, cudaStream_t s);
cudaError_t ep_peer_wait_launch(const uint32_t* flags, int n, const uint32_t* epoch_p, int* status,
                                long long budget_cycles, cudaStream_t s);
// Regions q0 .. q0 + nq - 1 (slots from region q0 on): rows past counts[q] get empty slots.
cudaError_t ep_peer_mask_launch(int32_t* slots, const int32_t* counts, int q0, int nq, int Tm, int K, cudaStream_t s);
// Receiver: the weighted sums of rows [0, nq * Tm) of regions q0 .. q0 + nq - 1
// (row r: region q0 + r / Tm, row r % Tm) stored into the sources' ret_y, and
// their result flags raised.
// With local_ret non-null the sums go to local_ret [regions][Tm][H] (row j of
// region q at (q * Tm + j) * H) and no flag is raised.
cudaError_t ep_peer_combine_launch(const __nv_bfloat16* y, const int32_t* slot_row, int q0, int nq, int K, int H,
                                   int Tm, int me, const EpPeerPtrs& peers, const EpPeerLayout& L, int P,
                                   unsigned* counter, const uint32_t* epoch_p, int max_ctas, cudaStream_t s,
                                   __nv_bfloat16* local_ret = nullptr);

// counts[e] = offsets[e+1] - offsets[e]
cudaError_t offsets_to_counts_launch(const int32_t* offsets, int32_t* counts, int n, cudaStream_t s);
// offsets[0] = 0, offsets[i+1] = offsets[i] + counts[i] (n <= kMaxExperts)
cudaError_t counts_to_offsets_launch(const int32_t* counts, int32_t* offsets, int n, cudaStream_t s);
cudaError_t aggregate_launch(const __nv_bfloat16* expert_outputs, __nv_bfloat16* out, int top_k, long long tokens,
                             int hidden, cudaStream_t s);
cudaError_t swiglu_launch(const __nv_bfloat16* gate_up, __nv_bfloat16* out, long long rows, int n, cudaStream_t s);

// ----------------------------------------------------------------- weight packing
// gate_up [E, H, 2I] (gate columns first) -> [E, 2I, H] K-major with the
// 64-row interleave [gate 64 | up 64] per 128-row block.
cudaError_t pack_gate_up_nxd_launch(const __nv_bfloat16* in, __nv_bfloat16* out, int experts, int hidden,
                                    int inter, cudaStream_t s);
// gate_up [E, 2I, H] (HF layout) -> same packed layout (row permutation).
cudaError_t pack_gate_up_hf_launch(const __nv_bfloat16* in, __nv_bfloat16* out, int experts, int hidden, int inter,
                                   cudaStream_t s);
// [B, R, C] -> [B, C, R] (bf16); used for down_proj [E, I, H] -> [E, H, I].
cudaError_t transpose_launch(const __nv_bfloat16* in, __nv_bfloat16* out, int batch, int rows, int cols,
                             cudaStream_t s);

// ----------------------------------------------------------------- grouped GEMM (tcgen05)
enum Epilogue : int {
  kEpiSwiGLU = 0,     // bf16 [R, N/2] = silu(gate) * up on the packed gate/up layout
  kEpiScaleBf16 = 1,  // bf16 [R, N] = slot_weight[row_slot[r]] * acc
  kEpiStoreBf16 = 2,  // bf16 [R, N]
  kEpiStoreF32 = 3,   // f32  [R, N] (+ col_bias[N])
};

struct GroupedGemmParams {
  const int32_t* expert_offsets;  // [E+1] segment starts of each expert's rows; null: one segment
  int dense_rows;                 // expert_offsets null: every expert has dense_rows rows, expert e
                                  // starting at row e * dense_rows
  int weight_mod;                 // > 0: segment e uses weight block e % weight_mod (expert-parallel
                                  // segments ordered (source rank, local expert)); 0: block e
  int shared_a;                   // 1: every expert reads activation rows [0, dense_rows) (its
                                  // output rows stay [e * dense_rows, (e + 1) * dense_rows))
  int num_experts;
  int n;           // output features per expert (rows of one expert's packed weight)
  int k_blocks;    // 64-wide K blocks iterated
  int k_blocks_a;  // 64-wide K blocks in an activation row (k coordinate of A wraps modulo this)
  int epilogue;
  void* out;
  long long out_ld;           // elements
  const float* slot_weight;   // kEpiScaleBf16: weight of row r = slot_weight[row_slot[r]] ...
  const int32_t* row_slot;
  const float* row_weight;    // ... or row_weight[r] when given (permuted order, one coalesced load)
  int prefetch;               // K blocks of the next tile prefetched into L2 at each tile start (0: off)
  int stage_stores;           // rows schedule, bf16 outputs through a per-warp staging tile: bit 0 SwiGLU,
                              // bit 1 scaled/plain bf16 (whole-sector row stores instead of 16-byte pieces)
  // Gathered activations: when a_row_map is set, activation row r of the
  // grouped problem is row a_row_map[r] of a_ptr (row stride a_ld elements),
  // loaded by the producer warp instead of a TMA tile load: with
  // tma_gather4 != 0 by TMA tile::gather4 through the activation tensor map
  // (box one row high; each lane loads four rows), else with cp.async.
  const int32_t* a_row_map;
  const __nv_bfloat16* a_ptr;
  long long a_ld;
  int tma_gather4;
  const int32_t* out_row_map; // optional: output row of permuted row r
  const float* col_bias;      // kEpiStoreF32 optional
  int* status;
  int row_split;              // rows schedules: 0 every row; 1 each expert's whole blocks of 256 rows
                              // (the SM-pair kernel); 2 the rows past them (the 1-SM kernel)
  int balance_waves;          // weights schedule: tiles dealt evenly to ceil(tiles / waves) CTAs
};

// Tile shape choices exposed to the host.
enum GemmVariant : int {
  kRowsBN256 = 0,  // 128 rows x 256 features per tile (prefill)
  kRowsBN128 = 1,  // 128 rows x 128 features per tile
  kWeightsT16 = 2, // 128 features x 16 rows per tile (decode, swap-AB)
  kWeightsT32 = 3, // 128 features x 32 rows per tile
  kWeightsT64 = 4, // 128 features x 64 rows per tile
  kRows2BN256 = 5, // 256 rows x 256 features per tile on an SM pair (cta_group::2)
  kTokens2 = 6,    // 256 features x up to 256 rows per tile on an SM pair (swap-AB, N per tile)
};

// Builds a 2-D bf16 TMA descriptor with 128-byte swizzling over a row-major
// [rows, cols] tensor; box = 64 columns x box_rows rows.
bool make_tmap_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, int box_rows);

cudaError_t grouped_gemm_launch(int variant, const CUtensorMap& tmap_act, const CUtensorMap& tmap_w,
                                const GroupedGemmParams& p, int grid, cudaStream_t s);
int grouped_gemm_box_rows_act(int variant);
int grouped_gemm_box_rows_w(int variant);

int device_sm_count();

// Sets the calling thread's message returned by nkimoe_last_error().
void set_last_error(const char* msg);
// Shape rules of the MoE block entry points (sets the last error on failure).
int check_moe_shapes(long long T, long long H, long long I, long long E, long long K);

}  // namespace nkimoe
