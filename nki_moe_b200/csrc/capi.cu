// C ABI (include/nkimoe.h): argument checks, workspace carving, TMA
// descriptors and the launch sequence of the MoE block.
//
// Launch sequence of one block (all on the caller's stream, no host sync):
//   [router: logits -> softmax/top-k]  permute  gather  GEMM-1 (+SwiGLU)
//   GEMM-2 (+routing weight)  combine
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>

#include "kernels.h"
#include "nkimoe.h"

namespace nkimoe {

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define NKI_CUDA(call)                                                                      \
  do {                                                                                      \
    cudaError_t e_ = (call);                                                                \
    if (e_ != cudaSuccess) return fail(NKIMOE_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

#define NKI_REQUIRE(cond, code, ...)         \
  do {                                       \
    if (!(cond)) return fail(code, __VA_ARGS__); \
  } while (0)

std::atomic<int> g_schedule{0};      // 0 auto, 1 rows, 2 weights
// Optional CUDA events recorded between the stages of a block call (set by
// nkimoe_set_stage_events, per calling thread): stage i starts at event i.
thread_local cudaEvent_t g_stage_events[kNumStageEvents] = {};
thread_local int g_num_stage_events = 0;

// During stream capture the record must be an external event node to be
// replayed with the graph (a plain record would only become a dependency).
inline void mark(int stage, cudaStream_t s) {
  if (stage >= g_num_stage_events || !g_stage_events[stage]) return;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &cs);
  if (cs == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(g_stage_events[stage], s, cudaEventRecordExternal);
  else
    cudaEventRecord(g_stage_events[stage], s);
}
std::atomic<int> g_weights_rows{0};  // 0 auto, else 16/32/64
std::atomic<int> g_router_permutes{1};  // decode routers of 9-255 tokens also write the permutation
std::atomic<int> g_router_halves{1};   // tensor-core router: two CTAs per row block (experts split)
std::atomic<int> g_weights_balance{1};  // weights-schedule GEMMs: tiles dealt evenly over the waves
std::atomic<int> g_router{0};        // 0 auto, 1 CUDA-core split-K, 2 tensor-core split-fp32
std::atomic<int> g_router_fused{1};  // tensor-core router: summed logits in one kernel (0: GEMM partials)
std::atomic<int> g_stage_stores{3};  // rows-schedule epilogue staging: bit 0 SwiGLU, bit 1 scaled bf16
std::atomic<int> g_gather_fused{0};  // GEMM-1 gathers its rows itself: 1 cp.async, 2 TMA gather4
std::atomic<int> g_prefetch{0};      // L2 prefetch distance of the rows-schedule GEMMs, in k-blocks
std::atomic<int> g_pdl{1};           // programmatic dependent launch of the decode-path kernels
// Budget of the expert-parallel waits for peers, in SM clock cycles (~10 s at
// 2 GHz by default): a peer that has not reached the step by then is reported
// as a timeout in the status word.
std::atomic<long long> g_peer_wait_cycles{20000000000LL};
// Expert-parallel schedule: -1 auto (the default: copy engines from 1024
// tokens on, one block below), 0 one block after all rows arrived, 1
// overlapped with SM stores, 2 overlapped with copy engines; groups of remote
// regions (0 auto); the grid bound of the send and return kernels that run
// beside the expert GEMMs (0: the SM count).
std::atomic<int> g_ep_overlap{-1};
std::atomic<int> g_ep_groups{0};
std::atomic<int> g_ep_side_ctas{0};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
inline size_t round256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

struct WsLayout {
  size_t status, logits, partial, idx, w, offsets, row_token, row_slot, slot_row, row_weight, scratch, xy, h, total;
};

WsLayout ws_layout(long long T, long long H, long long I, long long E, long long K) {
  WsLayout L{};
  size_t o = 0;
  const long long TK = T * K;
  L.status = o; o += 256;
  L.logits = o; o += round256(sizeof(float) * T * E);
  long long splits = 3;  // partial logits: tensor-core planes, split-K router or decode router slices
  if (T > 0) {
    splits = std::max<long long>(splits, router_splits_for(static_cast<int>(T), static_cast<int>(H), static_cast<int>(E)));
    if (H % 128 == 0 && (T + 7) / 8 <= router_topk_max_groups())
      splits = std::max<long long>(splits, router_topk_slices(static_cast<int>(T), static_cast<int>(H), static_cast<int>(E)));
  }
  L.partial = o; o += round256(sizeof(float) * splits * T * E);
  L.idx = o; o += round256(sizeof(int32_t) * TK);
  L.w = o; o += round256(sizeof(float) * TK);
  L.offsets = o; o += round256(sizeof(int32_t) * (E + 1));
  L.row_token = o; o += round256(sizeof(int32_t) * TK);
  L.row_slot = o; o += round256(sizeof(int32_t) * TK);
  L.slot_row = o; o += round256(sizeof(int32_t) * TK);
  L.row_weight = o; o += round256(sizeof(float) * TK);
  L.scratch = o; o += round256(permute_scratch_bytes(T, static_cast<int>(K), static_cast<int>(E)));
  L.xy = o; o += round256(sizeof(uint16_t) * TK * H);
  L.h = o; o += round256(sizeof(uint16_t) * TK * I);
  L.total = o;
  return L;
}

int choose_variant(long long rows_total, long long E, long long N) {
  const int sched = g_schedule.load();
  const double avg = E > 0 ? static_cast<double>(rows_total) / static_cast<double>(E) : 0.0;
  const bool weights = sched == 2 || (sched == 0 && avg <= 48.0);
  if (weights) {
    int r = g_weights_rows.load();
    if (r == 0) r = avg <= 8.0 ? 16 : (avg <= 24.0 ? 32 : 64);
    return r == 16 ? kWeightsT16 : (r == 32 ? kWeightsT32 : kWeightsT64);
  }
  // the SM-pair schedule is selected only on request: measured slower than the
  // 1-SM schedule on B200 for these shapes (TMA completions in the pair run at
  // about a third of the 1-SM rate)
  if (N % 256 == 0 && (sched == 3 || sched == 5)) return kRows2BN256;
  if (N % 256 == 0 && sched == 4) return kTokens2;
  return (N % 256 == 0) ? kRowsBN256 : kRowsBN128;
}

// One grouped GEMM: act [act_rows, kd] x w [E*N, kd]^T per expert segment.
// kd_act: K of an activation row; the weight row holds kd >= kd_act and the
// activation K coordinate wraps modulo kd_act (split-fp32 router: kd = 3 kd_act).
// offsets == nullptr: one dense segment of act_rows rows.
int run_gemm(const void* act, long long act_rows, const void* w, long long E, long long N, long long kd,
             const int32_t* offsets, int epilogue, void* out, long long out_ld, const float* slot_w,
             const int32_t* row_slot, const int32_t* out_row_map, const float* col_bias, int* status,
             cudaStream_t s, long long kd_act = 0, bool shared_a = false, const float* row_weight = nullptr,
             long long weight_experts = 0, int weight_mod = 0, const int32_t* a_row_map = nullptr,
             long long problem_rows = 0, long long choose_rows = 0, long long choose_experts = 0) {
  if (act_rows == 0) return NKIMOE_OK;
  if (kd_act == 0) kd_act = kd;
  // with shared activation rows every expert has act_rows rows; with gathered
  // rows the problem has problem_rows rows taken from the act_rows of `act`
  const long long rows_total = a_row_map ? problem_rows : (shared_a ? act_rows * E : act_rows);
  // a GEMM over part of a routing's experts takes the schedule of the whole
  int variant = choose_variant(choose_rows ? choose_rows : rows_total, choose_experts ? choose_experts : E, N);
  // the SM-pair kernels load A by TMA tiles only; the tokens kernel has no fp32 epilogue
  if ((variant == kRows2BN256 || variant == kTokens2) && (a_row_map || epilogue == kEpiStoreF32))
    variant = kRowsBN256;
  // the tokens kernel stores 16-byte vectors of an output row
  if (variant == kTokens2 && (reinterpret_cast<uintptr_t>(out) % 16 != 0 || out_ld % 8 != 0)) variant = kRowsBN256;
  // gathered rows by TMA gather4 read the activation map one row per box row
  const bool gather4 = a_row_map && g_gather_fused.load() == 2;
  CUtensorMap ta, tw;
  NKI_REQUIRE(make_tmap_bf16(&ta, act, act_rows, kd_act, gather4 ? 1 : grouped_gemm_box_rows_act(variant)),
              NKIMOE_ERR_CUDA,
              "cuTensorMapEncodeTiled failed for the activation operand");
  if (weight_experts == 0) weight_experts = E;
  NKI_REQUIRE(make_tmap_bf16(&tw, w, weight_experts * N, kd, grouped_gemm_box_rows_w(variant)), NKIMOE_ERR_CUDA,
              "cuTensorMapEncodeTiled failed for the weight operand");
  GroupedGemmParams p{};
  p.expert_offsets = offsets;
  p.dense_rows = static_cast<int>(act_rows);
  p.num_experts = static_cast<int>(E);
  p.n = static_cast<int>(N);
  p.k_blocks = static_cast<int>(kd / 64);
  p.k_blocks_a = static_cast<int>(kd_act / 64);
  p.shared_a = shared_a ? 1 : 0;
  p.weight_mod = weight_mod;
  p.a_row_map = a_row_map;
  p.a_ptr = static_cast<const __nv_bfloat16*>(act);
  p.a_ld = kd_act;
  p.tma_gather4 = gather4 ? 1 : 0;
  p.row_weight = row_weight;
  p.prefetch = g_prefetch.load();
  p.balance_waves = g_weights_balance.load();
  p.stage_stores = g_stage_stores.load();
  p.epilogue = epilogue;
  p.out = out;
  p.out_ld = out_ld;
  p.slot_weight = slot_w;
  p.row_slot = row_slot;
  p.out_row_map = out_row_map;
  p.col_bias = col_bias;
  p.status = status;
  const bool pair = variant == kRows2BN256 || variant == kTokens2;
  const bool rows = variant == kRowsBN256 || variant == kRowsBN128 || pair;
  const long long rpt = pair ? 256 : grouped_gemm_box_rows_act(variant);
  const long long fpt = pair ? 256 : (rows ? grouped_gemm_box_rows_w(variant) : 128);
  const long long max_tiles = (rows_total / rpt + E) * (N / fpt);
  long long grid = std::min<long long>(max_tiles, device_sm_count());
  if (pair) grid = 2 * std::max<long long>(1, std::min<long long>(max_tiles, device_sm_count() / 2));
  // schedule 5: the SM pair over each expert's whole 256-row blocks (no padded
  // rows), then the 1-SM kernel over the rows past them
  const bool split = variant == kRows2BN256 && g_schedule.load() == 5 && !shared_a && offsets;
  if (split) p.row_split = 1;
  NKI_CUDA(grouped_gemm_launch(variant, ta, tw, p, static_cast<int>(std::max<long long>(grid, 1)), s));
  if (split) {
    const int v2 = kRowsBN256;
    NKI_REQUIRE(make_tmap_bf16(&ta, act, act_rows, kd_act, grouped_gemm_box_rows_act(v2)) &&
                    make_tmap_bf16(&tw, w, weight_experts * N, kd, grouped_gemm_box_rows_w(v2)),
                NKIMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the remainder rows' operands");
    p.row_split = 2;
    // at most one 128-row block of remainder per 128 rows and per expert
    const long long tiles2 = (std::min<long long>(rows_total, E * 255) / 128 + E) * (N / 256);
    const long long grid2 = std::max<long long>(1, std::min<long long>(tiles2, device_sm_count()));
    NKI_CUDA(grouped_gemm_launch(v2, ta, tw, p, static_cast<int>(grid2), s));
  }
  return NKIMOE_OK;
}

// The router of a T-token batch runs on the tensor cores (three-plane split of
// the fp32 weights) when the caller passes the planes and the batch is large
// enough, unless the "router" option forces one kind.
bool router_uses_tensor_cores(bool have_split, long long T, long long E) {
  const int mode = g_router.load();
  return have_split && E % 128 == 0 && (mode == 2 || (mode == 0 && T >= 256));
}

// logits -> (idx, w): CUDA-core split-K or tensor-core split-fp32 GEMM, then
// softmax/top-k/renormalise.
// With `perm`, a decode batch of one token group (8 tokens or fewer) also gets
// its permutation from the router's last CTA; *permuted then says so.
int router_impl(const void* x, const float* router_w, const float* router_bias, const void* router_w_split,
                int32_t* idx, float* w, long long T, long long H, long long E, long long K, char* base,
                const WsLayout& L, int* status, cudaStream_t s, const RouterPermOut* perm = nullptr,
                bool* permuted = nullptr) {
  if (permuted) *permuted = false;
  float* logits = reinterpret_cast<float*>(base + L.logits);
  const bool tensor = router_uses_tensor_cores(router_w_split != nullptr, T, E);
  mark(kStageRouter, s);
  if (tensor && g_router_fused.load() && router_tc_supported(T, static_cast<int>(H), static_cast<int>(E), false)) {
    // the three planes' logits summed in one tensor-core kernel (the same MMAs
    // and sums as the router GEMM + partials form below), then the top-k
    CUtensorMap tx, tw;
    const int ept = g_router_halves.load() ? 64 : 128;  // experts per CTA = rows of a plane's TMA box
    NKI_REQUIRE(make_tmap_bf16(&tx, x, T, H, 128) && make_tmap_bf16(&tw, router_w_split, 3 * E, H, ept),
                NKIMOE_ERR_CUDA, "cuTensorMapEncodeTiled failed for the router operands");
    NKI_CUDA(router_tc_launch(tx, tw, nullptr, nullptr, 0, 0.f, nullptr, router_bias, logits, T, static_cast<int>(H),
                              status, s, ept));
    mark(kStageTopk, s);
    NKI_CUDA(topk_softmax_partials_launch(logits, 1, nullptr, nullptr, static_cast<int>(T), static_cast<int>(E),
                                          static_cast<int>(K), idx, w, s));
  } else if (tensor) {
    // the three bf16 planes are three "experts" over the same activation rows;
    // their fp32 partial logits [3][T][E] are added (hi + mid + lo) by top-k
    float* partial = reinterpret_cast<float*>(base + L.partial);
    int rc = run_gemm(x, T, router_w_split, 3, E, H, nullptr, kEpiStoreF32, partial, E, nullptr, nullptr, nullptr,
                      nullptr, status, s, H, true);
    if (rc != NKIMOE_OK) return rc;
    mark(kStageTopk, s);
    NKI_CUDA(topk_softmax_partials_launch(partial, 3, router_bias, logits, static_cast<int>(T), static_cast<int>(E),
                                          static_cast<int>(K), idx, w, s));
  } else if (router_topk_fused_supported(static_cast<int>(H), static_cast<int>(E), static_cast<int>(K)) && T > 8 &&
             T < 256) {
    // several token groups: 8-CTA clusters (faster than the split router
    // there); the grid's last CTA writes the permutation too (one counter in
    // the status block after the status word, cleared by every caller)
    const bool fuse_perm = perm && permuted && g_router_permutes.load() &&
                           router_topk_cluster_permutes(static_cast<int>(T), static_cast<int>(K));
    NKI_CUDA(router_topk_cluster_launch(static_cast<const __nv_bfloat16*>(x), router_w, router_bias, logits,
                                        static_cast<int>(T), static_cast<int>(H), static_cast<int>(E),
                                        static_cast<int>(K), idx, w, s, reinterpret_cast<int*>(base + L.status + 64),
                                        fuse_perm ? perm : nullptr));
    if (fuse_perm) *permuted = true;
    mark(kStageTopk, s);
  } else if (router_topk_fused_supported(static_cast<int>(H), static_cast<int>(E), static_cast<int>(K)) &&
             (T + 7) / 8 <= router_topk_max_groups()) {
    // logits and top-k in one launch; the top-k stage marker follows it.  Its
    // per-group counters sit in the status block after the status word, which
    // every caller clears (256 bytes) before the block.
    const bool fuse_perm = perm && permuted && router_topk_fused_permutes(static_cast<int>(T));
    NKI_CUDA(router_topk_fused_launch(static_cast<const __nv_bfloat16*>(x), router_w, router_bias, logits,
                                      static_cast<int>(T), static_cast<int>(H), static_cast<int>(E),
                                      static_cast<int>(K), idx, w, reinterpret_cast<float*>(base + L.partial),
                                      reinterpret_cast<int*>(base + L.status + 64), s, fuse_perm ? perm : nullptr));
    if (fuse_perm) *permuted = true;
    mark(kStageTopk, s);
  } else {
    float* partial = reinterpret_cast<float*>(base + L.partial);
    const int splits = router_splits_for(static_cast<int>(T), static_cast<int>(H), static_cast<int>(E));
    NKI_CUDA(router_splitk_launch(static_cast<const __nv_bfloat16*>(x), router_w, partial, static_cast<int>(T),
                                  static_cast<int>(H), static_cast<int>(E), splits, s));
    mark(kStageTopk, s);
    NKI_CUDA(topk_softmax_partials_launch(partial, splits, router_bias, logits, static_cast<int>(T),
                                          static_cast<int>(E), static_cast<int>(K), idx, w, s));
  }
  return NKIMOE_OK;
}

// Expert-parallel receiver: instead of writing `out`, the block's final sum of
// each row goes straight to the row's source rank (ep_peer.cu).
struct PeerCombine {
  EpPeerPtrs peers;
  EpPeerLayout L;
  int P, me, Tm;
  int q0, nq;      // the rows are those of regions q0 .. q0 + nq - 1
  int max_ctas;    // grid bound of the return kernel (0: none)
  unsigned* counter;
  const uint32_t* epoch_p;
};

// The decoder's residual add + RMSNorm after the block (qwen_with_nki.py:447-454):
// residual_out = residual + block output; out = rmsnorm(residual_out) * w.
struct FusedNorm {
  const void* residual;
  void* residual_out;
  const void* w;
  int w_dtype;
  float eps;
  void* out;
};

// The expert FFNs of a given routing over a workspace (ws_layout), in phases
// so that a caller can put other work between them: prep (permutation and row
// gather), GEMMs over a range of experts, finish (combine).
struct ExpertsRun {
  const void* x;
  const void* w13;
  const void* w2;
  const void* idx;
  int idx_dtype;
  const float* topk_w;
  long long T, H, I, E, K;
  char* base;
  WsLayout L;
  int* status;
};

ExpertsRun experts_run(const void* x, const void* w13, const void* w2, const void* idx, int idx_dtype,
                       const float* topk_w, long long T, long long H, long long I, long long E, long long K, void* ws,
                       int* status_word) {
  ExpertsRun r{x, w13, w2, idx, idx_dtype, topk_w, T, H, I, E, K, static_cast<char*>(ws), ws_layout(T, H, I, E, K),
               nullptr};
  r.status = status_word ? status_word : reinterpret_cast<int*>(r.base + r.L.status);
  return r;
}

int experts_prep(const ExpertsRun& r, cudaStream_t s, bool permuted, bool marks) {
  if (r.T == 0) return NKIMOE_OK;
  const WsLayout& L = r.L;
  int32_t* offsets = reinterpret_cast<int32_t*>(r.base + L.offsets);
  int32_t* row_token = reinterpret_cast<int32_t*>(r.base + L.row_token);
  if (marks) mark(kStagePermute, s);
  if (!permuted)  // else the router's last CTA has written the permutation
    NKI_CUDA(permute_launch(r.idx, r.idx_dtype, static_cast<int>(r.T), static_cast<int>(r.K), static_cast<int>(r.E),
                            row_token, reinterpret_cast<int32_t*>(r.base + L.row_slot),
                            reinterpret_cast<int32_t*>(r.base + L.slot_row), offsets, r.base + L.scratch, r.status, s,
                            r.topk_w, reinterpret_cast<float*>(r.base + L.row_weight)));
  if (marks) mark(kStageGather, s);
  if (!g_gather_fused.load())
    NKI_CUDA(gather_rows_launch(static_cast<const __nv_bfloat16*>(r.x), row_token, offsets, static_cast<int>(r.E),
                                reinterpret_cast<__nv_bfloat16*>(r.base + L.xy), r.T * r.K, static_cast<int>(r.H), s));
  return NKIMOE_OK;
}

// GEMM-1 (+SwiGLU) and GEMM-2 (+routing weight) of experts [e_lo, e_hi).  The
// tile schedule is the one the whole routing would get.
int experts_gemms(const ExpertsRun& r, long long e_lo, long long e_hi, cudaStream_t s, bool marks) {
  if (r.T == 0 || e_hi <= e_lo) return NKIMOE_OK;
  const WsLayout& L = r.L;
  const long long TK = r.T * r.K, H = r.H, I = r.I, E = e_hi - e_lo;
  const int32_t* offsets = reinterpret_cast<const int32_t*>(r.base + L.offsets) + e_lo;
  const char* w13 = static_cast<const char*>(r.w13) + sizeof(uint16_t) * e_lo * 2 * I * H;
  const char* w2 = static_cast<const char*>(r.w2) + sizeof(uint16_t) * e_lo * H * I;
  __nv_bfloat16* xy = reinterpret_cast<__nv_bfloat16*>(r.base + L.xy);
  __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(r.base + L.h);
  int rc;
  if (marks) mark(kStageGemm1, s);
  if (g_gather_fused.load()) {
    // GEMM-1 gathers its activation rows (x[row_token[r]]) in its producer warp
    rc = run_gemm(r.x, r.T, w13, E, 2 * I, H, offsets, kEpiSwiGLU, h, I, nullptr, nullptr, nullptr, nullptr, r.status,
                  s, 0, false, nullptr, 0, 0, reinterpret_cast<const int32_t*>(r.base + L.row_token), TK, TK, r.E);
  } else {
    rc = run_gemm(xy, TK, w13, E, 2 * I, H, offsets, kEpiSwiGLU, h, I, nullptr, nullptr, nullptr, nullptr, r.status, s,
                  0, false, nullptr, 0, 0, nullptr, 0, TK, r.E);
  }
  if (rc != NKIMOE_OK) return rc;
  if (marks) mark(kStageGemm2, s);
  return run_gemm(h, TK, w2, E, H, I, offsets, kEpiScaleBf16, xy, H, r.topk_w,
                  reinterpret_cast<const int32_t*>(r.base + L.row_slot), nullptr, nullptr, r.status, s, 0, false,
                  reinterpret_cast<const float*>(r.base + L.row_weight), 0, 0, nullptr, 0, TK, r.E);
}

int experts_finish(const ExpertsRun& r, void* out, const PeerCombine* pc, const FusedNorm* fn, cudaStream_t s,
                   bool marks) {
  if (r.T == 0) return NKIMOE_OK;
  const WsLayout& L = r.L;
  const long long T = r.T, K = r.K, H = r.H;
  const __nv_bfloat16* xy = reinterpret_cast<const __nv_bfloat16*>(r.base + L.xy);
  const int32_t* slot_row = reinterpret_cast<const int32_t*>(r.base + L.slot_row);
  __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(r.base + L.h);
  if (marks) mark(kStageCombine, s);
  if (pc) {
    NKI_CUDA(ep_peer_combine_launch(xy, slot_row, pc->q0, pc->nq, static_cast<int>(K), static_cast<int>(H), pc->Tm,
                                    pc->me, pc->peers, pc->L, pc->P, pc->counter, pc->epoch_p, pc->max_ctas, s));
  } else if (fn && combine_add_rmsnorm_supported(T, static_cast<int>(H))) {
    // few rows: the combine and the next residual add + norm in one kernel
    NKI_CUDA(combine_add_rmsnorm_launch(xy, slot_row, static_cast<int>(K),
                                        static_cast<const __nv_bfloat16*>(fn->residual),
                                        static_cast<__nv_bfloat16*>(fn->residual_out), fn->w, fn->w_dtype,
                                        static_cast<__nv_bfloat16*>(fn->out), T, static_cast<int>(H), fn->eps, s));
  } else if (fn) {
    // the block output goes through the SwiGLU buffer, free after GEMM-2
    NKI_CUDA(combine_launch(xy, slot_row, nullptr, h, static_cast<int>(T), static_cast<int>(K), static_cast<int>(H),
                            s));
    NKI_CUDA(add_rmsnorm_launch(h, fn->residual, fn->residual_out, fn->w, fn->w_dtype, fn->out, T,
                                static_cast<int>(H), fn->eps, s));
  } else {
    NKI_CUDA(combine_launch(xy, slot_row, nullptr, static_cast<__nv_bfloat16*>(out), static_cast<int>(T),
                            static_cast<int>(K), static_cast<int>(H), s));
  }
  if (marks) mark(kStageEnd, s);
  return NKIMOE_OK;
}

int experts_impl(const void* x, const void* w13, const void* w2, const void* idx, int idx_dtype, const float* topk_w,
                 void* out, long long T, long long H, long long I, long long E, long long K, void* ws, size_t ws_bytes,
                 cudaStream_t s, const PeerCombine* pc = nullptr, int* status_word = nullptr,
                 const FusedNorm* fn = nullptr, bool permuted = false) {
  (void)ws_bytes;
  if (T == 0) return NKIMOE_OK;
  const ExpertsRun r = experts_run(x, w13, w2, idx, idx_dtype, topk_w, T, H, I, E, K, ws, status_word);
  int rc = experts_prep(r, s, permuted, true);
  if (rc == NKIMOE_OK) rc = experts_gemms(r, 0, E, s, true);
  if (rc == NKIMOE_OK) rc = experts_finish(r, out, pc, fn, s, true);
  return rc;
}

// Workspace of nkimoe_ep_peer_forward: routing of the local tokens, the
// (token, rank) sort, the row map of the final sum, completion counters, then
// the receiver's expert blocks.  The one-block schedule runs one block over
// all P * max_tokens region rows; the overlapped schedule runs one block over
// the rank's own tokens (their own-expert slots in self_idx / self_w) and one
// per group of remote regions.  The workspace holds the larger of the two.
struct PeerWs {
  size_t route, disp, slot_in, slot_out, counters, self_idx, self_w, idx_v, recv;
  // copy-engine schedule: outgoing rows per destination and returned sums per region
  size_t stage_x, stage_slots, stage_w, stage_counts, ret_stage, total;
};

size_t ep_dispatch_ws_bytes(long long T, long long P);

// Regions q >= 1 cut into `groups` groups of consecutive regions, nearly equal,
// the later groups taking the remainder: group g is [q0(g), q0(g + 1)).
inline long long group_q0(long long P, long long groups, long long g) {
  const long long n = P - 1, base = n / groups, extra = n % groups;
  return 1 + g * base + std::max<long long>(0, g - (groups - extra));
}

size_t overlapped_recv_bytes(long long T, long long H, long long I, long long El, long long K, long long P,
                             long long Tm, long long groups) {
  size_t o = round256(ws_layout(T, H, I, El, K).total);  // own tokens
  for (long long g = 0; g < groups; ++g) {
    const long long nq = group_q0(P, groups, g + 1) - group_q0(P, groups, g);
    o += round256(ws_layout(nq * Tm, H, I, El, K).total);
  }
  return o;
}

// El: expert slots per rank (E / P, or more with hot-expert replicas).
PeerWs peer_ws(long long T, long long H, long long I, long long E, long long K, long long P, long long Tm,
               long long El) {
  PeerWs W{};
  size_t o = 0;
  W.route = o; o += round256(ws_layout(T, H, I, E, K).offsets);  // status, logits, partials, idx, w
  W.disp = o; o += round256(ep_dispatch_ws_bytes(T, P));
  W.slot_in = o; o += round256(sizeof(int32_t) * T * P);
  W.slot_out = o; o += round256(sizeof(int32_t) * T * P);
  W.counters = o; o += 256;
  W.self_idx = o; o += round256(sizeof(int32_t) * T * K);
  W.self_w = o; o += round256(sizeof(float) * T * K);
  W.idx_v = o; o += round256(sizeof(int32_t) * T * K);
  W.recv = o;
  size_t recv = ws_layout(P * Tm, H, I, El, K).total;
  for (long long g = 1; g < P; ++g) recv = std::max(recv, overlapped_recv_bytes(T, H, I, El, K, P, Tm, g));
  o += round256(recv);
  W.stage_x = o; o += round256(sizeof(uint16_t) * P * Tm * H);
  W.stage_slots = o; o += round256(sizeof(int32_t) * P * Tm * K);
  W.stage_w = o; o += round256(sizeof(float) * P * Tm * K);
  W.stage_counts = o; o += 256;
  W.ret_stage = o; o += round256(sizeof(uint16_t) * P * Tm * H);
  W.total = o;
  return W;
}

}  // namespace

int check_moe_shapes(long long T, long long H, long long I, long long E, long long K) {
  NKI_REQUIRE(T >= 0 && H > 0 && I > 0 && E > 0 && K > 0, NKIMOE_ERR_INVALID_ARG, "non-positive dimension");
  NKI_REQUIRE(E <= kMaxExperts, NKIMOE_ERR_UNSUPPORTED, "num_experts %lld > %d", E, kMaxExperts);
  NKI_REQUIRE(K <= 32 && K <= E, NKIMOE_ERR_UNSUPPORTED, "top_k %lld must be <= 32 and <= num_experts", K);
  NKI_REQUIRE(H % 128 == 0, NKIMOE_ERR_UNSUPPORTED, "hidden %lld must be a multiple of 128", H);
  NKI_REQUIRE(I % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "intermediate %lld must be a multiple of 64", I);
  NKI_REQUIRE(T * K < (1LL << 31), NKIMOE_ERR_UNSUPPORTED, "T*K too large");
  return NKIMOE_OK;
}

bool make_tmap_bf16(CUtensorMap* map, const void* base, long long rows, long long cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn || rows <= 0 || cols <= 0 || (cols * 2) % 16 != 0 || !aligned16(base)) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

void set_last_error(const char* msg) { g_err = msg ? msg : ""; }

namespace {
size_t ep_dispatch_ws_bytes(long long T, long long P) {
  const long long TP = T * P;
  return 256 + round256(sizeof(int32_t) * (P + 1)) + 3 * round256(sizeof(int32_t) * TP) +
         round256(permute_scratch_bytes(T, static_cast<int>(P), static_cast<int>(P)));
}
}  // namespace

int device_sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = n > 0 ? n : 148;
  }
  return counts[dev];
}

bool pdl_enabled() { return g_pdl.load() != 0; }

}  // namespace nkimoe

using namespace nkimoe;

namespace {

int moe_block_impl(const void* x, const float* router_w, const float* router_bias, const void* router_w_split,
                   const void* w13, const void* w2, void* out, int32_t* topk_idx_out, float* topk_w_out, int64_t T,
                   int64_t H, int64_t I, int64_t E, int64_t K, void* workspace, size_t workspace_bytes, void* stream,
                   const FusedNorm* fn, bool keep_status = false) {
  int rc = check_moe_shapes(T, H, I, E, K);
  if (rc != NKIMOE_OK) return rc;
  NKI_REQUIRE(E <= 256, NKIMOE_ERR_UNSUPPORTED, "router top-k supports up to 256 experts");
  const size_t need = nkimoe_moe_workspace_bytes(T, H, I, E, K);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  NKI_REQUIRE(aligned16(workspace), NKIMOE_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
  const cudaStream_t s = as_stream(stream);
  if (keep_status)  // a later chunk of one call: the status word keeps the earlier chunks' faults
    NKI_CUDA(cudaMemsetAsync(static_cast<char*>(workspace) + sizeof(int), 0, 256 - sizeof(int), s));
  else
    NKI_CUDA(cudaMemsetAsync(workspace, 0, 256, s));  // status word and router counters
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && router_w && w13 && w2 && (out || fn), NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(x) && aligned16(router_w) && aligned16(w13) && aligned16(w2) && (fn || aligned16(out)),
              NKIMOE_ERR_INVALID_ARG, "x, weights and out must be 16-byte aligned");
  if (fn) {
    NKI_REQUIRE(fn->residual && fn->residual_out && fn->w && fn->out, NKIMOE_ERR_INVALID_ARG, "null pointer");
    NKI_REQUIRE(aligned16(fn->residual) && aligned16(fn->residual_out) && aligned16(fn->w) && aligned16(fn->out),
                NKIMOE_ERR_INVALID_ARG, "residual, norm weight and outputs must be 16-byte aligned");
    NKI_REQUIRE(fn->w_dtype == NKIMOE_F32 || fn->w_dtype == NKIMOE_BF16, NKIMOE_ERR_INVALID_ARG,
                "bad norm weight dtype");
    NKI_REQUIRE(H % 8 == 0, NKIMOE_ERR_UNSUPPORTED, "hidden must be a multiple of 8");
  }
  NKI_REQUIRE(!router_w_split || aligned16(router_w_split), NKIMOE_ERR_INVALID_ARG, "router_w_split misaligned");
  const WsLayout L = ws_layout(T, H, I, E, K);
  char* base = static_cast<char*>(workspace);
  int32_t* idx = topk_idx_out ? topk_idx_out : reinterpret_cast<int32_t*>(base + L.idx);
  float* w = topk_w_out ? topk_w_out : reinterpret_cast<float*>(base + L.w);
  int* status = reinterpret_cast<int*>(base + L.status);
  const RouterPermOut perm{reinterpret_cast<int32_t*>(base + L.row_token), reinterpret_cast<int32_t*>(base + L.row_slot),
                           reinterpret_cast<int32_t*>(base + L.slot_row), reinterpret_cast<int32_t*>(base + L.offsets),
                           reinterpret_cast<float*>(base + L.row_weight), status};
  bool permuted = false;
  rc = router_impl(x, router_w, router_bias, router_w_split, idx, w, T, H, E, K, base, L, status, s, &perm,
                   &permuted);
  if (rc != NKIMOE_OK) return rc;
  return experts_impl(x, w13, w2, idx, NKIMOE_I32, w, out, T, H, I, E, K, workspace, workspace_bytes, s, nullptr,
                      nullptr, fn, permuted);
}

// ---- block on host buffers: token chunks whose copies overlap the block ----
constexpr int kMaxHostChunks = 16;

// Token chunks of a host-buffer block call.  A chunk is cut only where every
// chunk takes the path the whole batch takes: the tensor-core router (256
// tokens or more) and the tile-rows GEMM schedule (more than 48 rows per expert
// on average, the auto schedule's threshold), so the output is the whole-batch
// block's bit for bit: each row's router dot products, expert GEMM sums and
// slot combine do not depend on the other rows of its batch.  requested <= 0:
// half the batch (measured at 8192 tokens: 2 chunks 1.64 ms, 3 chunks 1.72, 4
// chunks 1.83, one 1.98 with the copies serialised; every chunk re-reads the
// expert weights).  The last chunk takes the remainder, merged into the one
// before it when shorter than the minimum.
struct HostChunks {
  long long len, count, longest;
};

HostChunks host_chunks(long long T, long long E, long long K, bool have_split, long long requested) {
  HostChunks c{T, 1, T};
  if (T <= 0 || !router_uses_tensor_cores(have_split, T, E)) return c;
  long long min_len = 256;
  const int sched = g_schedule.load();
  if (sched == 2) return c;  // weight-streaming schedule: its tile height follows the batch
  if (sched == 0) {
    if (T * K <= 48 * E) return c;
    min_len = std::max(min_len, (48 * E) / K + 1);
  }
  long long len = requested > 0 ? requested : (T + 1) / 2;
  len = std::max({len, min_len, (T + kMaxHostChunks - 1) / kMaxHostChunks});
  if (len >= T) return c;
  long long n = (T + len - 1) / len;
  if (T - (n - 1) * len < min_len) --n;  // a short tail joins the chunk before it
  c.len = len;
  c.count = n;
  c.longest = T - (n - 1) * len;
  if (c.longest < len) c.longest = len;
  return c;
}

size_t host_stage_bytes(long long T, long long H) { return round256(sizeof(uint16_t) * T * H); }

// Block workspace of any chunk of a T-token batch: every region of the block
// workspace grows with the tokens except the router's partial logits (up to 8
// per logit, more per token for small batches), bounded here by 8 per logit.
size_t host_block_bytes(long long T, long long H, long long I, long long E, long long K) {
  return nkimoe_moe_workspace_bytes(T, H, I, E, K) + round256(sizeof(float) * 8 * T * E);
}

// Per device: a stream for host->device copies, one for device->host copies
// and the per-chunk events that order them against the caller's stream.  Per
// workspace: two slots of staging rows used by alternate calls, each with the
// events that say when its last user is done with it (input rows read by the
// block, output rows copied back), so that one call's copies overlap the
// block of the call before or after it.
struct HostSlots {
  unsigned calls = 0;
  long long last_tokens = -1;  // batch size of the previous call (its staging layout)
  cudaEvent_t x_free[2] = {}, out_free[2] = {};
};
struct HostCopyStreams {
  bool ready = false;
  cudaStream_t in = nullptr, out = nullptr;
  cudaEvent_t in_done[kMaxHostChunks] = {}, blk_done[kMaxHostChunks] = {};
  std::map<void*, HostSlots> slots;
};
constexpr int kHostMaxDevices = 64;
std::mutex g_host_mu[kHostMaxDevices];
HostCopyStreams g_host[kHostMaxDevices];

int host_streams_init(HostCopyStreams& h) {
  if (h.ready) return NKIMOE_OK;
  NKI_CUDA(cudaStreamCreateWithFlags(&h.in, cudaStreamNonBlocking));
  NKI_CUDA(cudaStreamCreateWithFlags(&h.out, cudaStreamNonBlocking));
  for (int i = 0; i < kMaxHostChunks; ++i) {
    NKI_CUDA(cudaEventCreateWithFlags(&h.in_done[i], cudaEventDisableTiming));
    NKI_CUDA(cudaEventCreateWithFlags(&h.blk_done[i], cudaEventDisableTiming));
  }
  h.ready = true;
  return NKIMOE_OK;
}

int host_slots_for(HostCopyStreams& h, void* workspace, HostSlots** out) {
  auto it = h.slots.find(workspace);
  if (it == h.slots.end()) {
    HostSlots hs;
    for (int i = 0; i < 2; ++i) {
      NKI_CUDA(cudaEventCreateWithFlags(&hs.x_free[i], cudaEventDisableTiming));
      NKI_CUDA(cudaEventCreateWithFlags(&hs.out_free[i], cudaEventDisableTiming));
    }
    it = h.slots.emplace(workspace, hs).first;
  }
  *out = &it->second;
  return NKIMOE_OK;
}

// Per device: the side stream of the expert-parallel block (sends and returns
// beside the expert GEMMs) and the events that fork it from and join it to
// the caller's stream.  Calls on one device share it (and its lock).
constexpr int kEpMaxDevices = 64;
struct EpSideStream {
  bool ready = false;
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr, group[kMaxPeers] = {};
};
std::mutex g_ep_mu[kEpMaxDevices];
EpSideStream g_ep[kEpMaxDevices];

int ep_side_init(EpSideStream& es) {
  if (es.ready) return NKIMOE_OK;
  NKI_CUDA(cudaStreamCreateWithFlags(&es.side, cudaStreamNonBlocking));
  NKI_CUDA(cudaEventCreateWithFlags(&es.fork, cudaEventDisableTiming));
  NKI_CUDA(cudaEventCreateWithFlags(&es.join, cudaEventDisableTiming));
  for (int g = 0; g < kMaxPeers; ++g) NKI_CUDA(cudaEventCreateWithFlags(&es.group[g], cudaEventDisableTiming));
  es.ready = true;
  return NKIMOE_OK;
}

}  // namespace

extern "C" {

int nkimoe_version(void) { return 1; }

int nkimoe_set_stage_events(void* const* events, int count) {
  if (count < 0 || count > kNumStageEvents || (count > 0 && !events))
    return fail(NKIMOE_ERR_INVALID_ARG, "stage events: 0..%d events", kNumStageEvents);
  for (int i = 0; i < kNumStageEvents; ++i)
    g_stage_events[i] = i < count ? static_cast<cudaEvent_t>(events[i]) : nullptr;
  g_num_stage_events = count;
  return NKIMOE_OK;
}

const char* nkimoe_last_error(void) { return g_err.c_str(); }

int nkimoe_set_option(const char* name, long long value) {
  if (!name) return fail(NKIMOE_ERR_INVALID_ARG, "null option name");
  const std::string n(name);
  if (n == "gemm_schedule" && value >= 0 && value <= 5) {
    g_schedule = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "weights_rows" && (value == 0 || value == 16 || value == 32 || value == 64)) {
    g_weights_rows = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "router_permutes" && (value == 0 || value == 1)) {
    g_router_permutes = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "router_halves" && (value == 0 || value == 1)) {
    g_router_halves = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "weights_balance" && (value == 0 || value == 1)) {
    g_weights_balance = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "epilogue_staging" && value >= 0 && value <= 3) {
    g_stage_stores = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "gather_fused" && value >= 0 && value <= 2) {
    g_gather_fused = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "prefetch" && value >= 0 && value <= 16) {
    g_prefetch = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "pdl" && (value == 0 || value == 1)) {
    g_pdl = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "router" && value >= 0 && value <= 2) {
    g_router = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "router_fused" && (value == 0 || value == 1)) {
    g_router_fused = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "peer_wait_cycles" && value >= 1000 && value <= 1000000000000LL) {
    g_peer_wait_cycles = value;
    return NKIMOE_OK;
  }
  if (n == "ep_overlap" && value >= -1 && value <= 2) {
    g_ep_overlap = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "ep_groups" && value >= 0 && value < kMaxPeers) {
    g_ep_groups = static_cast<int>(value);
    return NKIMOE_OK;
  }
  if (n == "ep_side_ctas" && value >= 0 && value <= 4096) {
    g_ep_side_ctas = static_cast<int>(value);
    return NKIMOE_OK;
  }
  return fail(NKIMOE_ERR_INVALID_ARG, "unknown option %s=%lld", name, value);
}

int nkimoe_rmsnorm(const void* x, int x_dtype, const void* weight, int w_dtype, void* out, int out_dtype,
                   int64_t rows, int64_t hidden, float eps, void* stream) {
  NKI_REQUIRE(rows >= 0 && hidden > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(hidden % 8 == 0, NKIMOE_ERR_UNSUPPORTED, "hidden %lld must be a multiple of 8", (long long)hidden);
  if (rows == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && weight && out, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(out), NKIMOE_ERR_INVALID_ARG,
              "pointers must be 16-byte aligned");
  cudaError_t e = rmsnorm_launch(x, x_dtype, weight, w_dtype, out, out_dtype, rows, static_cast<int>(hidden), eps,
                                 as_stream(stream));
  NKI_REQUIRE(e != cudaErrorInvalidValue, NKIMOE_ERR_INVALID_ARG, "unsupported dtype combination %d/%d/%d", x_dtype,
              w_dtype, out_dtype);
  NKI_CUDA(e);
  return NKIMOE_OK;
}

int nkimoe_add_rmsnorm(const void* x, const void* residual, void* residual_out, const void* weight, int w_dtype,
                       void* out, int64_t rows, int64_t hidden, float eps, void* stream) {
  NKI_REQUIRE(rows >= 0 && hidden > 0 && hidden % 8 == 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  if (rows == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && residual && residual_out && weight && out, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(x) && aligned16(residual) && aligned16(residual_out) && aligned16(weight) && aligned16(out),
              NKIMOE_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  cudaError_t e = add_rmsnorm_launch(x, residual, residual_out, weight, w_dtype, out, rows, static_cast<int>(hidden),
                                     eps, as_stream(stream));
  NKI_REQUIRE(e != cudaErrorInvalidValue, NKIMOE_ERR_INVALID_ARG, "unsupported weight dtype %d", w_dtype);
  NKI_CUDA(e);
  return NKIMOE_OK;
}

int nkimoe_qk_norm_rope(const void* qkv_in, void* qkv_out, const void* q_weight, const void* k_weight, int w_dtype,
                        const int64_t* positions, int64_t tokens, int n_heads, int n_kv_heads, int head_dim,
                        float rope_theta, float eps, void* stream) {
  NKI_REQUIRE(tokens >= 0 && n_heads > 0 && n_kv_heads >= 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(head_dim == 128, NKIMOE_ERR_UNSUPPORTED, "head_dim %d (only 128 is supported)", head_dim);
  NKI_REQUIRE(w_dtype == NKIMOE_F32 || w_dtype == NKIMOE_BF16, NKIMOE_ERR_INVALID_ARG, "bad weight dtype");
  if (tokens == 0) return NKIMOE_OK;
  NKI_REQUIRE(qkv_in && qkv_out && q_weight && k_weight && positions, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(qkv_in) && aligned16(qkv_out), NKIMOE_ERR_INVALID_ARG, "qkv must be 16-byte aligned");
  NKI_CUDA(qk_norm_rope_launch(qkv_in, qkv_out, q_weight, k_weight, w_dtype,
                               reinterpret_cast<const long long*>(positions), tokens, n_heads, n_kv_heads, head_dim,
                               rope_theta, eps, as_stream(stream)));
  return NKIMOE_OK;
}

size_t nkimoe_decode_attention_workspace_bytes(int64_t batch, int n_heads, int n_kv_heads, int head_dim,
                                               int64_t max_seq) {
  if (batch < 0 || n_heads <= 0 || n_kv_heads <= 0 || head_dim != 128 || max_seq <= 0) return 0;
  return decode_attention_workspace_bytes(batch, n_heads, n_kv_heads, static_cast<int>(max_seq));
}

int nkimoe_decode_attention(const void* qkv, const void* q_weight, const void* k_weight, int w_dtype,
                            const int64_t* positions, int64_t pos_stride, void* k_cache, void* v_cache, void* out,
                            int64_t batch, int n_heads, int n_kv_heads, int head_dim, int64_t max_seq,
                            float rope_theta, float eps, float scale, void* workspace, size_t workspace_bytes,
                            void* stream) {
  NKI_REQUIRE(batch >= 0 && n_heads > 0 && n_kv_heads > 0 && max_seq > 0 && pos_stride >= 0,
              NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(head_dim == 128, NKIMOE_ERR_UNSUPPORTED, "head_dim %d (only 128 is supported)", head_dim);
  NKI_REQUIRE(n_heads % n_kv_heads == 0, NKIMOE_ERR_INVALID_ARG, "n_heads %d is not a multiple of n_kv_heads %d",
              n_heads, n_kv_heads);
  NKI_REQUIRE(n_heads / n_kv_heads <= 16, NKIMOE_ERR_UNSUPPORTED, "more than 16 query heads per kv head");
  NKI_REQUIRE(max_seq <= (1LL << 30) && batch <= 65535 && n_kv_heads <= 65535, NKIMOE_ERR_UNSUPPORTED,
              "shape too large");
  NKI_REQUIRE(w_dtype == NKIMOE_F32 || w_dtype == NKIMOE_BF16, NKIMOE_ERR_INVALID_ARG, "bad weight dtype");
  if (batch == 0) return NKIMOE_OK;
  NKI_REQUIRE(qkv && q_weight && k_weight && positions && k_cache && v_cache && out && workspace,
              NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(qkv) && aligned16(k_cache) && aligned16(v_cache) && aligned16(out) && aligned16(workspace),
              NKIMOE_ERR_INVALID_ARG, "qkv, caches, out and workspace must be 16-byte aligned");
  const size_t need = decode_attention_workspace_bytes(batch, n_heads, n_kv_heads, static_cast<int>(max_seq));
  NKI_REQUIRE(workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu bytes < %zu", workspace_bytes, need);
  NKI_CUDA(decode_attention_launch(static_cast<const __nv_bfloat16*>(qkv), q_weight, k_weight, w_dtype,
                                   reinterpret_cast<const long long*>(positions), pos_stride,
                                   static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache),
                                   static_cast<__nv_bfloat16*>(out), static_cast<int>(batch), n_heads, n_kv_heads,
                                   static_cast<int>(max_seq), rope_theta, eps, scale, workspace, as_stream(stream)));
  return NKIMOE_OK;
}

int nkimoe_skinny_linear(const void* x, const void* w, void* y, int64_t M, int64_t N, int64_t K, void* stream) {
  NKI_REQUIRE(M >= 0 && N >= 0 && K > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(M <= 16, NKIMOE_ERR_UNSUPPORTED, "skinny_linear takes at most 16 rows (%lld)", (long long)M);
  NKI_REQUIRE(N % 16 == 0 && K % 32 == 0, NKIMOE_ERR_UNSUPPORTED, "N %% 16 and K %% 32 must be 0 (N=%lld K=%lld)",
              (long long)N, (long long)K);
  NKI_REQUIRE(N / 16 <= 0x7fffffffLL && K <= 0x7fffffffLL, NKIMOE_ERR_UNSUPPORTED, "shape too large");
  if (M == 0 || N == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && w && y, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(x) && aligned16(w) && aligned16(y), NKIMOE_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  NKI_CUDA(skinny_linear_launch(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
                                static_cast<__nv_bfloat16*>(y), static_cast<int>(M), static_cast<int>(N),
                                static_cast<int>(K), as_stream(stream)));
  return NKIMOE_OK;
}

int nkimoe_router_logits(const void* x, const float* router_w, const float* router_bias, float* logits, int64_t T,
                         int64_t H, int64_t E, void* stream) {
  NKI_REQUIRE(T >= 0 && H > 0 && E > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(H % 32 == 0, NKIMOE_ERR_UNSUPPORTED, "hidden %lld must be a multiple of 32", (long long)H);
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && router_w && logits, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(x) && aligned16(router_w), NKIMOE_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  NKI_CUDA(router_logits_simt_launch(static_cast<const __nv_bfloat16*>(x), router_w, router_bias, logits,
                                     static_cast<int>(T), static_cast<int>(H), static_cast<int>(E), as_stream(stream)));
  return NKIMOE_OK;
}

int nkimoe_router_split(const float* router_w, void* router_w_split, int64_t E, int64_t H, void* stream) {
  NKI_REQUIRE(router_w && router_w_split && E > 0 && H > 0, NKIMOE_ERR_INVALID_ARG, "bad argument");
  NKI_REQUIRE(H % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "hidden must be a multiple of 64");
  NKI_CUDA(router_split_launch(router_w, static_cast<__nv_bfloat16*>(router_w_split), static_cast<int>(E),
                               static_cast<int>(H), as_stream(stream)));
  return NKIMOE_OK;
}

int nkimoe_topk_softmax(const float* logits, int64_t T, int64_t E, int64_t K, int32_t* topk_idx, float* topk_w,
                        void* stream) {
  NKI_REQUIRE(T >= 0 && E > 0 && K > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(E <= 256 && K <= 32 && K <= E, NKIMOE_ERR_UNSUPPORTED, "E <= 256 and K <= min(32, E) required");
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(logits && topk_idx && topk_w, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_CUDA(topk_softmax_launch(logits, static_cast<int>(T), static_cast<int>(E), static_cast<int>(K), topk_idx, topk_w,
                               as_stream(stream)));
  return NKIMOE_OK;
}

size_t nkimoe_permute_workspace_bytes(int64_t T, int64_t K, int64_t E) {
  return 256 + permute_scratch_bytes(T, static_cast<int>(K), static_cast<int>(E));
}

int nkimoe_permute(const void* topk_idx, int idx_dtype, int64_t T, int64_t K, int64_t E, int32_t* row_token,
                   int32_t* row_slot, int32_t* slot_row, int32_t* expert_offsets, void* workspace,
                   size_t workspace_bytes, void* stream) {
  NKI_REQUIRE(T >= 0 && K > 0 && E > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(E <= kMaxExperts, NKIMOE_ERR_UNSUPPORTED, "num_experts > %d", kMaxExperts);
  NKI_REQUIRE(idx_dtype == NKIMOE_I32 || idx_dtype == NKIMOE_I64, NKIMOE_ERR_INVALID_ARG, "idx dtype must be I32/I64");
  NKI_REQUIRE(workspace_bytes >= nkimoe_permute_workspace_bytes(T, K, E), NKIMOE_ERR_WORKSPACE,
              "workspace %zu < %zu", workspace_bytes, nkimoe_permute_workspace_bytes(T, K, E));
  NKI_REQUIRE(expert_offsets && workspace, NKIMOE_ERR_INVALID_ARG, "null pointer");
  const cudaStream_t s = as_stream(stream);
  int* status = static_cast<int*>(workspace);
  NKI_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s));
  if (T > 0) NKI_REQUIRE(topk_idx && row_token && row_slot && slot_row, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_CUDA(permute_launch(topk_idx, idx_dtype, static_cast<int>(T), static_cast<int>(K), static_cast<int>(E), row_token,
                          row_slot, slot_row, expert_offsets, static_cast<char*>(workspace) + 256, status, s));
  return NKIMOE_OK;
}

int nkimoe_pack_gate_up(const void* gate_up, int layout, void* w13, int64_t E, int64_t H, int64_t I, void* stream) {
  NKI_REQUIRE(gate_up && w13 && E > 0 && H > 0 && I > 0, NKIMOE_ERR_INVALID_ARG, "bad argument");
  NKI_REQUIRE(I % 64 == 0 && H % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "I and H must be multiples of 64");
  NKI_REQUIRE(aligned16(gate_up) && aligned16(w13), NKIMOE_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  const auto* in = static_cast<const __nv_bfloat16*>(gate_up);
  auto* out = static_cast<__nv_bfloat16*>(w13);
  if (layout == NKIMOE_LAYOUT_NXD) {
    NKI_CUDA(pack_gate_up_nxd_launch(in, out, static_cast<int>(E), static_cast<int>(H), static_cast<int>(I),
                                     as_stream(stream)));
  } else if (layout == NKIMOE_LAYOUT_HF) {
    NKI_CUDA(pack_gate_up_hf_launch(in, out, static_cast<int>(E), static_cast<int>(H), static_cast<int>(I),
                                    as_stream(stream)));
  } else {
    return fail(NKIMOE_ERR_INVALID_ARG, "unknown layout %d", layout);
  }
  return NKIMOE_OK;
}

int nkimoe_pack_down(const void* down, int layout, void* w2, int64_t E, int64_t H, int64_t I, void* stream) {
  NKI_REQUIRE(down && w2 && E > 0 && H > 0 && I > 0, NKIMOE_ERR_INVALID_ARG, "bad argument");
  NKI_REQUIRE(I % 64 == 0 && H % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "I and H must be multiples of 64");
  if (layout == NKIMOE_LAYOUT_NXD) {
    NKI_CUDA(transpose_launch(static_cast<const __nv_bfloat16*>(down), static_cast<__nv_bfloat16*>(w2),
                              static_cast<int>(E), static_cast<int>(I), static_cast<int>(H), as_stream(stream)));
  } else if (layout == NKIMOE_LAYOUT_HF) {
    NKI_CUDA(cudaMemcpyAsync(w2, down, sizeof(uint16_t) * E * H * I, cudaMemcpyDeviceToDevice, as_stream(stream)));
  } else {
    return fail(NKIMOE_ERR_INVALID_ARG, "unknown layout %d", layout);
  }
  return NKIMOE_OK;
}

size_t nkimoe_moe_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K) {
  return ws_layout(T, H, I, E, K).total;
}

int nkimoe_moe_experts(const void* x, const void* w13, const void* w2, const void* topk_idx, int idx_dtype,
                       const float* topk_w, void* out, int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                       void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_moe_shapes(T, H, I, E, K);
  if (rc != NKIMOE_OK) return rc;
  NKI_REQUIRE(idx_dtype == NKIMOE_I32 || idx_dtype == NKIMOE_I64, NKIMOE_ERR_INVALID_ARG, "idx dtype must be I32/I64");
  const size_t need = nkimoe_moe_workspace_bytes(T, H, I, E, K);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  NKI_REQUIRE(aligned16(workspace), NKIMOE_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
  const cudaStream_t s = as_stream(stream);
  NKI_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && w13 && w2 && topk_idx && topk_w && out, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(x) && aligned16(w13) && aligned16(w2) && aligned16(out), NKIMOE_ERR_INVALID_ARG,
              "x, weights and out must be 16-byte aligned");
  return experts_impl(x, w13, w2, topk_idx, idx_dtype, topk_w, out, T, H, I, E, K, workspace, workspace_bytes, s);
}

int nkimoe_moe_block(const void* x, const float* router_w, const float* router_bias, const void* router_w_split,
                     const void* w13, const void* w2, void* out, int32_t* topk_idx_out, float* topk_w_out, int64_t T,
                     int64_t H, int64_t I, int64_t E, int64_t K, void* workspace, size_t workspace_bytes,
                     void* stream) {
  return moe_block_impl(x, router_w, router_bias, router_w_split, w13, w2, out, topk_idx_out, topk_w_out, T, H, I, E,
                        K, workspace, workspace_bytes, stream, nullptr);
}

int nkimoe_moe_block_add_rmsnorm(const void* x, const float* router_w, const float* router_bias,
                                 const void* router_w_split, const void* w13, const void* w2, const void* residual,
                                 void* residual_out, const void* norm_w, int norm_w_dtype, float eps, void* norm_out,
                                 int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I,
                                 int64_t E, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  const FusedNorm fn{residual, residual_out, norm_w, norm_w_dtype, eps, norm_out};
  return moe_block_impl(x, router_w, router_bias, router_w_split, w13, w2, nullptr, topk_idx_out, topk_w_out, T, H,
                        I, E, K, workspace, workspace_bytes, stream, &fn);
}

size_t nkimoe_moe_block_rmsnorm_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K) {
  if (T < 0 || H <= 0) return 0;
  return nkimoe_moe_workspace_bytes(T, H, I, E, K) + round256(sizeof(uint16_t) * T * H);
}

int nkimoe_moe_block_rmsnorm(const void* h, const void* norm_w, int norm_w_dtype, float eps, void* x_out,
                             const float* router_w, const float* router_bias, const void* router_w_split,
                             const void* w13, const void* w2, void* out, int32_t* topk_idx_out, float* topk_w_out,
                             int64_t T, int64_t H, int64_t I, int64_t E, int64_t K, void* workspace,
                             size_t workspace_bytes, void* stream) {
  int rc = check_moe_shapes(T, H, I, E, K);
  if (rc != NKIMOE_OK) return rc;
  NKI_REQUIRE(E <= 256, NKIMOE_ERR_UNSUPPORTED, "router top-k supports up to 256 experts");
  const size_t need = nkimoe_moe_block_rmsnorm_workspace_bytes(T, H, I, E, K);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  NKI_REQUIRE(aligned16(workspace), NKIMOE_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
  NKI_REQUIRE(norm_w_dtype == NKIMOE_F32 || norm_w_dtype == NKIMOE_BF16, NKIMOE_ERR_INVALID_ARG,
              "norm weight dtype must be F32 or BF16");
  const cudaStream_t s = as_stream(stream);
  NKI_CUDA(cudaMemsetAsync(workspace, 0, 256, s));  // status word and router counters
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(h && norm_w && router_w && w13 && w2 && out, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(h) && aligned16(norm_w) && aligned16(router_w) && aligned16(w13) && aligned16(w2) &&
                  aligned16(out) && (!x_out || aligned16(x_out)) && (!router_w_split || aligned16(router_w_split)),
              NKIMOE_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  const WsLayout L = ws_layout(T, H, I, E, K);
  char* base = static_cast<char*>(workspace);
  void* x = x_out ? x_out : base + nkimoe_moe_workspace_bytes(T, H, I, E, K);
  int32_t* idx = topk_idx_out ? topk_idx_out : reinterpret_cast<int32_t*>(base + L.idx);
  float* w = topk_w_out ? topk_w_out : reinterpret_cast<float*>(base + L.w);
  int* status = reinterpret_cast<int*>(base + L.status);
  // Prefill batches on the tensor-core router: the norm and the logits in one
  // kernel that writes the normalised rows once, then the top-k.  (Up to 512 rows
  // RMSNorm runs its one-CTA-per-row kernel, whose reduction order differs, so
  // the fused kernel starts above that and stays bit-identical to the unfused
  // calls.)  Otherwise: the RMSNorm kernel, then the router.
  const bool fused = router_uses_tensor_cores(router_w_split != nullptr, T, E) && g_router_fused.load() && T > 512 &&
                     router_tc_supported(T, static_cast<int>(H), static_cast<int>(E), true);
  if (fused) {
    CUtensorMap tw;
    const int ept = g_router_halves.load() ? 64 : 128;  // experts per CTA = rows of a plane's TMA box
    NKI_REQUIRE(make_tmap_bf16(&tw, router_w_split, 3 * E, H, ept), NKIMOE_ERR_CUDA,
                "cuTensorMapEncodeTiled failed for the router planes");
    float* logits = reinterpret_cast<float*>(base + L.logits);
    mark(kStageRouter, s);
    NKI_CUDA(router_tc_launch(tw, tw, static_cast<const __nv_bfloat16*>(h), norm_w, norm_w_dtype, eps,
                              static_cast<__nv_bfloat16*>(x), router_bias, logits, T, static_cast<int>(H), status, s,
                              ept));
    mark(kStageTopk, s);
    NKI_CUDA(topk_softmax_partials_launch(logits, 1, nullptr, nullptr, static_cast<int>(T), static_cast<int>(E),
                                          static_cast<int>(K), idx, w, s));
  } else {
    NKI_CUDA(rmsnorm_launch(h, NKIMOE_BF16, norm_w, norm_w_dtype, x, NKIMOE_BF16, T, static_cast<int>(H), eps, s));
    rc = router_impl(x, router_w, router_bias, router_w_split, idx, w, T, H, E, K, base, L, status, s);
    if (rc != NKIMOE_OK) return rc;
  }
  return experts_impl(x, w13, w2, idx, NKIMOE_I32, w, out, T, H, I, E, K, workspace, workspace_bytes, s);
}

size_t nkimoe_moe_block_host_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K) {
  if (T < 0 || H <= 0 || E <= 0) return 0;
  return host_block_bytes(T, H, I, E, K) + 4 * host_stage_bytes(T, H);  // two slots of input + output rows
}

int nkimoe_moe_block_host_plan(int64_t T, int64_t E, int64_t K, int have_router_split, int64_t chunk_tokens,
                               int64_t* chunk_len, int64_t* chunk_count) {
  NKI_REQUIRE(T >= 0 && E > 0 && K > 0 && chunk_len && chunk_count, NKIMOE_ERR_INVALID_ARG, "bad plan arguments");
  const HostChunks ch = host_chunks(T, E, K, have_router_split != 0, chunk_tokens);
  *chunk_len = ch.len;
  *chunk_count = ch.count;
  return NKIMOE_OK;
}

int nkimoe_moe_block_host(const void* x_host, const float* router_w, const float* router_bias,
                          const void* router_w_split, const void* w13, const void* w2, void* out_host,
                          int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E,
                          int64_t K, int64_t chunk_tokens, void* workspace, size_t workspace_bytes, void* done_event,
                          void* stream) {
  int rc = check_moe_shapes(T, H, I, E, K);
  if (rc != NKIMOE_OK) return rc;
  const size_t need = nkimoe_moe_block_host_workspace_bytes(T, H, I, E, K);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  NKI_REQUIRE(aligned16(workspace), NKIMOE_ERR_INVALID_ARG, "workspace must be 16-byte aligned");
  const cudaStream_t s = as_stream(stream);
  const cudaEvent_t done = static_cast<cudaEvent_t>(done_event);
  if (T == 0) {
    NKI_CUDA(cudaMemsetAsync(workspace, 0, 256, s));
    if (done) NKI_CUDA(cudaEventRecord(done, s));
    return NKIMOE_OK;
  }
  NKI_REQUIRE(x_host && out_host, NKIMOE_ERR_INVALID_ARG, "null host buffer");
  const HostChunks ch = host_chunks(T, E, K, router_w_split != nullptr, chunk_tokens);
  int dev = 0;
  NKI_CUDA(cudaGetDevice(&dev));
  NKI_REQUIRE(dev >= 0 && dev < kHostMaxDevices, NKIMOE_ERR_UNSUPPORTED, "device %d", dev);
  std::lock_guard<std::mutex> lock(g_host_mu[dev]);
  HostCopyStreams& hs = g_host[dev];
  rc = host_streams_init(hs);
  if (rc != NKIMOE_OK) return rc;
  HostSlots* sl = nullptr;
  rc = host_slots_for(hs, workspace, &sl);
  if (rc != NKIMOE_OK) return rc;
  const unsigned k = sl->calls++ & 1u;
  // the block workspace (status word first), then this call's slot of staging rows
  const size_t blk_bytes = host_block_bytes(T, H, I, E, K);
  char* xs = static_cast<char*>(workspace) + blk_bytes + k * 2 * host_stage_bytes(T, H);
  char* os = xs + host_stage_bytes(T, H);
  const size_t row_bytes = sizeof(uint16_t) * static_cast<size_t>(H);
  // The staging slots sit after the block workspace, whose size follows T, so
  // with the same T a slot only overlaps its own previous use.  When T changes
  // this call's rows may lie on the previous calls' block scratch or staging
  // rows: its copies in then wait for both slots' blocks and copies back, and
  // its block for both copies back.
  if (sl->last_tokens >= 0 && sl->last_tokens != T) {
    for (int i = 0; i < 2; ++i) {
      NKI_CUDA(cudaStreamWaitEvent(hs.in, sl->x_free[i], 0));
      NKI_CUDA(cudaStreamWaitEvent(hs.in, sl->out_free[i], 0));
      NKI_CUDA(cudaStreamWaitEvent(s, sl->out_free[i], 0));
    }
  }
  sl->last_tokens = T;
  // input rows: after the block of this slot's previous call has read them
  NKI_CUDA(cudaStreamWaitEvent(hs.in, sl->x_free[k], 0));
  for (long long c = 0; c < ch.count; ++c) {
    const long long t0 = c * ch.len, n = c + 1 < ch.count ? ch.len : T - t0;
    NKI_CUDA(cudaMemcpyAsync(xs + t0 * row_bytes, static_cast<const char*>(x_host) + t0 * row_bytes, n * row_bytes,
                             cudaMemcpyHostToDevice, hs.in));
    NKI_CUDA(cudaEventRecord(hs.in_done[c], hs.in));
  }
  // output rows: after this slot's previous copy back to the host
  NKI_CUDA(cudaStreamWaitEvent(s, sl->out_free[k], 0));
  for (long long c = 0; c < ch.count; ++c) {
    const long long t0 = c * ch.len, n = c + 1 < ch.count ? ch.len : T - t0;
    NKI_CUDA(cudaStreamWaitEvent(s, hs.in_done[c], 0));
    rc = moe_block_impl(xs + t0 * row_bytes, router_w, router_bias, router_w_split, w13, w2, os + t0 * row_bytes,
                        topk_idx_out ? topk_idx_out + t0 * K : nullptr, topk_w_out ? topk_w_out + t0 * K : nullptr, n,
                        H, I, E, K, workspace, blk_bytes, s, nullptr, c > 0);
    if (rc != NKIMOE_OK) return rc;
    NKI_CUDA(cudaEventRecord(hs.blk_done[c], s));
    NKI_CUDA(cudaStreamWaitEvent(hs.out, hs.blk_done[c], 0));
    NKI_CUDA(cudaMemcpyAsync(static_cast<char*>(out_host) + t0 * row_bytes, os + t0 * row_bytes, n * row_bytes,
                             cudaMemcpyDeviceToHost, hs.out));
  }
  NKI_CUDA(cudaEventRecord(sl->x_free[k], s));
  NKI_CUDA(cudaEventRecord(sl->out_free[k], hs.out));
  if (done) {
    // the caller waits on done_event; the stream goes on to its next work
    NKI_CUDA(cudaEventRecord(done, hs.out));
  } else {
    // the caller's stream completes with the last copy to the host
    NKI_CUDA(cudaStreamWaitEvent(s, sl->out_free[k], 0));
  }
  return NKIMOE_OK;
}

int nkimoe_read_status(void* workspace, void* stream, int* status_out) {
  NKI_REQUIRE(workspace, NKIMOE_ERR_INVALID_ARG, "null workspace");
  const cudaStream_t s = as_stream(stream);
  int v = 0;
  NKI_CUDA(cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
  NKI_CUDA(cudaStreamSynchronize(s));
  NKI_CUDA(cudaMemsetAsync(workspace, 0, sizeof(int), s));
  if (status_out) *status_out = v;
  if (v != 0) return fail(NKIMOE_ERR_DEVICE, "device status 0x%x (1 = wait timeout, 2 = expert id or cache position out of range)", v);
  return NKIMOE_OK;
}

int nkimoe_grouped_gemm(const void* a, const void* w_packed, const int32_t* expert_offsets, const int32_t* out_row_map,
                        void* out, int64_t M, int64_t N, int64_t Kd, int64_t E, int* status, void* stream) {
  NKI_REQUIRE(M >= 0 && N > 0 && Kd > 0 && E > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  NKI_REQUIRE(E <= kMaxExperts, NKIMOE_ERR_UNSUPPORTED, "num_experts > %d", kMaxExperts);
  NKI_REQUIRE(N % 128 == 0 && Kd % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "N %% 128 == 0 and K %% 64 == 0 required");
  if (M == 0) return NKIMOE_OK;
  NKI_REQUIRE(a && w_packed && expert_offsets && out, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_REQUIRE(aligned16(a) && aligned16(w_packed) && aligned16(out), NKIMOE_ERR_INVALID_ARG,
              "pointers must be 16-byte aligned");
  return run_gemm(a, M, w_packed, E, N, Kd, expert_offsets, kEpiStoreBf16, out, N, nullptr, nullptr, out_row_map,
                  nullptr, status, as_stream(stream));
}

int nkimoe_swiglu(const void* gate_up, void* out, int64_t M, int64_t N, void* stream) {
  NKI_REQUIRE(M >= 0 && N > 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  if (M == 0) return NKIMOE_OK;
  NKI_REQUIRE(gate_up && out, NKIMOE_ERR_INVALID_ARG, "null pointer");
  NKI_CUDA(swiglu_launch(static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), M,
                         static_cast<int>(N), as_stream(stream)));
  return NKIMOE_OK;
}

int nkimoe_aggregate(const void* expert_outputs, void* out, int64_t K, int64_t T, int64_t H, void* stream) {
  NKI_REQUIRE(K > 0 && T >= 0 && H > 0 && H % 8 == 0, NKIMOE_ERR_INVALID_ARG, "bad shape");
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(expert_outputs && out && aligned16(expert_outputs) && aligned16(out), NKIMOE_ERR_INVALID_ARG,
              "null or unaligned pointer");
  NKI_CUDA(aggregate_launch(static_cast<const __nv_bfloat16*>(expert_outputs), static_cast<__nv_bfloat16*>(out),
                            static_cast<int>(K), T, static_cast<int>(H), as_stream(stream)));
  return NKIMOE_OK;
}

// ------------------------------------------------------------ expert parallel pieces

size_t nkimoe_route_workspace_bytes(int64_t T, int64_t H, int64_t E, int64_t K) {
  const WsLayout L = ws_layout(T, H, 64, E, K);
  return L.partial + round256(sizeof(float) * std::max<long long>(
                                  T > 0 ? router_splits_for(static_cast<int>(T), static_cast<int>(H),
                                                            static_cast<int>(E))
                                        : 1,
                                  3) *
                              T * E);
}

int nkimoe_route(const void* x, const float* router_w, const float* router_bias, const void* router_w_split,
                 int32_t* topk_idx, float* topk_w, int64_t T, int64_t H, int64_t E, int64_t K, void* workspace,
                 size_t workspace_bytes, void* stream) {
  NKI_REQUIRE(T >= 0 && H > 0 && E > 0 && K > 0 && K <= 32 && K <= E && E <= 256, NKIMOE_ERR_UNSUPPORTED,
              "route: bad shape");
  NKI_REQUIRE(H % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "hidden must be a multiple of 64");
  const size_t need = nkimoe_route_workspace_bytes(T, H, E, K);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  const cudaStream_t s = as_stream(stream);
  NKI_CUDA(cudaMemsetAsync(workspace, 0, 256, s));  // status word and router counters
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(x && router_w && topk_idx && topk_w && aligned16(x) && aligned16(router_w), NKIMOE_ERR_INVALID_ARG,
              "null or misaligned pointer");
  const WsLayout L = ws_layout(T, H, 64, E, K);
  char* base = static_cast<char*>(workspace);
  return router_impl(x, router_w, router_bias, router_w_split, topk_idx, topk_w, T, H, E, K, base, L,
                     reinterpret_cast<int*>(base + L.status), s);
}

size_t nkimoe_dispatch_workspace_bytes(int64_t T, int64_t K, int64_t E) {
  const long long TK = T * K;
  return 256 + round256(sizeof(int32_t) * (E + 1)) + 2 * round256(sizeof(int32_t) * TK) +
         round256(permute_scratch_bytes(T, static_cast<int>(K), static_cast<int>(E)));
}

int nkimoe_dispatch(const void* x, const void* topk_idx, int idx_dtype, const float* topk_w, int64_t T, int64_t H,
                    int64_t E, int64_t K, void* x_perm, float* row_weight, int32_t* slot_row, int32_t* expert_counts,
                    void* workspace, size_t workspace_bytes, void* stream) {
  NKI_REQUIRE(T >= 0 && H > 0 && E > 0 && K > 0 && E <= kMaxExperts && H % 8 == 0, NKIMOE_ERR_UNSUPPORTED,
              "dispatch: bad shape");
  NKI_REQUIRE(idx_dtype == NKIMOE_I32 || idx_dtype == NKIMOE_I64, NKIMOE_ERR_INVALID_ARG, "idx dtype must be I32/I64");
  const size_t need = nkimoe_dispatch_workspace_bytes(T, K, E);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  const cudaStream_t s = as_stream(stream);
  char* base = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(base);
  NKI_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s));
  int32_t* offsets = reinterpret_cast<int32_t*>(base + 256);
  if (T == 0) {
    NKI_CUDA(cudaMemsetAsync(expert_counts, 0, sizeof(int32_t) * E, s));
    return NKIMOE_OK;
  }
  NKI_REQUIRE(x && topk_idx && topk_w && x_perm && row_weight && slot_row && expert_counts && aligned16(x) &&
                  aligned16(x_perm),
              NKIMOE_ERR_INVALID_ARG, "null or misaligned pointer");
  const long long TK = T * K;
  int32_t* row_token = offsets + round256(sizeof(int32_t) * (E + 1)) / sizeof(int32_t);
  int32_t* row_slot = row_token + round256(sizeof(int32_t) * TK) / sizeof(int32_t);
  void* scratch = row_slot + round256(sizeof(int32_t) * TK) / sizeof(int32_t);
  NKI_CUDA(permute_launch(topk_idx, idx_dtype, static_cast<int>(T), static_cast<int>(K), static_cast<int>(E), row_token,
                          row_slot, slot_row, offsets, scratch, status, s, topk_w, row_weight));
  NKI_CUDA(gather_rows_launch(static_cast<const __nv_bfloat16*>(x), row_token, offsets, static_cast<int>(E),
                              static_cast<__nv_bfloat16*>(x_perm), TK, static_cast<int>(H), s));
  NKI_CUDA(offsets_to_counts_launch(offsets, expert_counts, static_cast<int>(E), s));
  return NKIMOE_OK;
}

size_t nkimoe_segment_experts_workspace_bytes(int64_t rows, int64_t I, int64_t segments) {
  return 256 + round256(sizeof(int32_t) * (segments + 1)) + round256(sizeof(uint16_t) * rows * I);
}

int nkimoe_segment_experts(const void* a, const float* row_weight, const int32_t* segment_counts, int64_t segments,
                           int64_t experts_per_group, const void* w13, const void* w2, void* y, int64_t rows,
                           int64_t H, int64_t I, void* workspace, size_t workspace_bytes, void* stream) {
  NKI_REQUIRE(rows >= 0 && H > 0 && I > 0 && segments > 0 && segments <= kMaxExperts && experts_per_group > 0,
              NKIMOE_ERR_UNSUPPORTED, "segment experts: bad shape");
  NKI_REQUIRE(H % 128 == 0 && I % 64 == 0, NKIMOE_ERR_UNSUPPORTED, "H %% 128 == 0 and I %% 64 == 0 required");
  const size_t need = nkimoe_segment_experts_workspace_bytes(rows, I, segments);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  const cudaStream_t s = as_stream(stream);
  char* base = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(base);
  NKI_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s));
  if (rows == 0) return NKIMOE_OK;
  NKI_REQUIRE(a && row_weight && segment_counts && w13 && w2 && y && aligned16(a) && aligned16(w13) && aligned16(w2) &&
                  aligned16(y),
              NKIMOE_ERR_INVALID_ARG, "null or misaligned pointer");
  int32_t* offsets = reinterpret_cast<int32_t*>(base + 256);
  __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(base + 256 + round256(sizeof(int32_t) * (segments + 1)));
  NKI_CUDA(counts_to_offsets_launch(segment_counts, offsets, static_cast<int>(segments), s));
  int rc = run_gemm(a, rows, w13, segments, 2 * I, H, offsets, kEpiSwiGLU, h, I, nullptr, nullptr, nullptr, nullptr,
                    status, s, 0, false, nullptr, experts_per_group, static_cast<int>(experts_per_group));
  if (rc != NKIMOE_OK) return rc;
  return run_gemm(h, rows, w2, segments, H, I, offsets, kEpiScaleBf16, y, H, nullptr, nullptr, nullptr, nullptr,
                  status, s, 0, false, row_weight, experts_per_group, static_cast<int>(experts_per_group));
}

size_t nkimoe_ep_dispatch_workspace_bytes(int64_t T, int64_t P) { return ep_dispatch_ws_bytes(T, P); }

int nkimoe_ep_dispatch(const void* x, const int32_t* topk_idx, const float* topk_w, int64_t T, int64_t H, int64_t K,
                       int64_t num_ranks, int64_t experts_per_rank, void* x_send, int32_t* slots_send,
                       float* weights_send, int32_t* rank_counts, int32_t* slot_row, void* workspace,
                       size_t workspace_bytes, void* stream) {
  const long long P = num_ranks, El = experts_per_rank;
  NKI_REQUIRE(T >= 0 && H > 0 && K > 0 && P > 0 && El > 0 && P <= kMaxExperts && H % 8 == 0,
              NKIMOE_ERR_UNSUPPORTED, "ep dispatch: bad shape");
  const size_t need = nkimoe_ep_dispatch_workspace_bytes(T, P);
  NKI_REQUIRE(workspace && workspace_bytes >= need, NKIMOE_ERR_WORKSPACE, "workspace %zu < %zu", workspace_bytes, need);
  const cudaStream_t s = as_stream(stream);
  char* base = static_cast<char*>(workspace);
  int* status = reinterpret_cast<int*>(base);
  NKI_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s));
  if (T == 0) {
    NKI_CUDA(cudaMemsetAsync(rank_counts, 0, sizeof(int32_t) * P, s));
    return NKIMOE_OK;
  }
  NKI_REQUIRE(x && topk_idx && topk_w && x_send && slots_send && weights_send && rank_counts && slot_row &&
                  aligned16(x) && aligned16(x_send),
              NKIMOE_ERR_INVALID_ARG, "null or misaligned pointer");
  const long long TP = T * P;
  int32_t* offsets = reinterpret_cast<int32_t*>(base + 256);
  int32_t* dest = offsets + round256(sizeof(int32_t) * (P + 1)) / sizeof(int32_t);
  int32_t* row_token = dest + round256(sizeof(int32_t) * TP) / sizeof(int32_t);
  int32_t* row_slot = row_token + round256(sizeof(int32_t) * TP) / sizeof(int32_t);
  void* scratch = row_slot + round256(sizeof(int32_t) * TP) / sizeof(int32_t);
  // (token, rank) pairs grouped by rank, tokens ascending: the permutation of
  // the [T, P] destination matrix with ranks as the sort keys
  NKI_CUDA(ep_dest_launch(topk_idx, static_cast<int>(T), static_cast<int>(K), static_cast<int>(P),
                          static_cast<int>(El), dest, s));
  NKI_CUDA(permute_launch(dest, NKIMOE_I32, static_cast<int>(T), static_cast<int>(P), static_cast<int>(P), row_token,
                          row_slot, slot_row, offsets, scratch, status, s));
  NKI_CUDA(gather_rows_launch(static_cast<const __nv_bfloat16*>(x), row_token, offsets, static_cast<int>(P),
                              static_cast<__nv_bfloat16*>(x_send), TP, static_cast<int>(H), s));
  NKI_CUDA(ep_slots_launch(topk_idx, topk_w, row_token, row_slot, offsets, TP, static_cast<int>(P),
                           static_cast<int>(K), static_cast<int>(El), slots_send, weights_send, s));
  NKI_CUDA(offsets_to_counts_launch(offsets, rank_counts, static_cast<int>(P), s));
  return NKIMOE_OK;
}

size_t nkimoe_ep_peer_buffer_bytes(int64_t num_ranks, int64_t max_tokens, int64_t H, int64_t K) {
  if (num_ranks <= 0 || max_tokens < 0 || H <= 0 || K <= 0) return 0;
  return ep_peer_layout(num_ranks, max_tokens, H, K).total;
}

int nkimoe_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  NKI_REQUIRE(bytes > 0 && ptr && ipc_handle, NKIMOE_ERR_INVALID_ARG, "peer alloc: bad arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == NKIMOE_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  NKI_CUDA(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaMemset(p, 0, bytes);  // epoch flags start at 0
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(NKIMOE_ERR_CUDA, "peer alloc: %s", cudaGetErrorString(e));
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return NKIMOE_OK;
}

int nkimoe_peer_open(const void* ipc_handle, void** ptr) {
  NKI_REQUIRE(ipc_handle && ptr, NKIMOE_ERR_INVALID_ARG, "peer open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  NKI_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return NKIMOE_OK;
}

int nkimoe_peer_close(void* ptr) {
  NKI_REQUIRE(ptr, NKIMOE_ERR_INVALID_ARG, "peer close: null pointer");
  NKI_CUDA(cudaIpcCloseMemHandle(ptr));
  return NKIMOE_OK;
}

int nkimoe_peer_free(void* ptr) {
  NKI_REQUIRE(ptr, NKIMOE_ERR_INVALID_ARG, "peer free: null pointer");
  NKI_CUDA(cudaFree(ptr));
  return NKIMOE_OK;
}

size_t nkimoe_ep_peer_workspace_bytes(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K, int64_t num_ranks,
                                      int64_t max_tokens) {
  if (num_ranks <= 0 || E % num_ranks != 0) return 0;
  return peer_ws(T, H, I, E, K, num_ranks, max_tokens, E / num_ranks).total;
}

size_t nkimoe_ep_peer_workspace_bytes_mapped(int64_t T, int64_t H, int64_t I, int64_t E, int64_t K,
                                             int64_t num_ranks, int64_t max_tokens, int64_t local_slots) {
  if (num_ranks <= 0 || local_slots <= 0 || local_slots > kMaxExperts) return 0;
  return peer_ws(T, H, I, E, K, num_ranks, max_tokens, local_slots).total;
}

int nkimoe_ep_peer_schedule(int64_t num_ranks, int64_t max_tokens) {
  const int schedule = g_ep_overlap.load();
  if (schedule >= 0) return schedule;
  return (num_ranks > 1 && num_ranks <= 4 && max_tokens >= 1024) ? 2 : 0;
}

// The expert-parallel block; El expert slots per rank, slot v on rank
// v / El.  Without expert_slots slot v is expert v (El = E / P); with them
// slot (t, k) of expert e goes to slot expert_slots[e * max_holders + t mod
// slot_counts[e]] (hot-expert replicas).
static int ep_peer_forward_impl(const void* x, const float* router_w, const float* router_bias,
                                const void* router_w_split, const void* w13_local, const void* w2_local, void* out,
                                int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E,
                                int64_t K, int64_t num_ranks, int64_t rank, int64_t max_tokens,
                                void* const* peer_buffers, uint32_t epoch, void* workspace, size_t workspace_bytes,
                                void* stream, long long El, const int32_t* expert_slots, const int32_t* slot_counts,
                                long long max_holders) {
  const long long P = num_ranks, Tm = max_tokens;
  int rc = check_moe_shapes(std::max<long long>(T, 1), H, I, E, K);
  if (rc != NKIMOE_OK) return rc;
  NKI_REQUIRE(P >= 1 && P <= kMaxPeers && rank >= 0 && rank < P && (expert_slots || E % P == 0),
              NKIMOE_ERR_UNSUPPORTED,
              "ep peer: need 1 <= ranks <= %d dividing the experts, 0 <= rank < ranks", kMaxPeers);
  NKI_REQUIRE(El >= 1 && El <= kMaxExperts && (!expert_slots || (slot_counts && max_holders >= 1 &&
                                                                  max_holders <= kMaxExperts)),
              NKIMOE_ERR_INVALID_ARG, "ep peer: bad expert slot map (%lld slots per rank, %lld holders)", El,
              max_holders);
  NKI_REQUIRE(T >= 0 && T <= Tm && P * Tm * K < (1LL << 31) && P * Tm * (H / 8) < (1LL << 31) && E <= 256,
              NKIMOE_ERR_UNSUPPORTED, "ep peer: tokens %lld exceed max_tokens %lld or the buffers are too large",
              static_cast<long long>(T), Tm);
  const PeerWs W = peer_ws(T, H, I, E, K, P, Tm, El);
  NKI_REQUIRE(workspace && workspace_bytes >= W.total && aligned16(workspace), NKIMOE_ERR_WORKSPACE,
              "workspace %zu < %zu", workspace_bytes, W.total);
  NKI_REQUIRE(peer_buffers && router_w && w13_local && w2_local && (T == 0 || (x && out)), NKIMOE_ERR_INVALID_ARG,
              "null pointer");
  EpPeerPtrs peers{};
  for (long long r = 0; r < P; ++r) {
    NKI_REQUIRE(peer_buffers[r] && (reinterpret_cast<uintptr_t>(peer_buffers[r]) & 255u) == 0,
                NKIMOE_ERR_INVALID_ARG, "peer buffer %lld null or not 256-byte aligned", r);
    peers.base[r] = static_cast<char*>(peer_buffers[r]);
  }
  NKI_REQUIRE(T == 0 || (aligned16(x) && aligned16(out)), NKIMOE_ERR_INVALID_ARG, "x and out must be 16-byte aligned");
  const cudaStream_t s = as_stream(stream);
  const EpPeerLayout PL = ep_peer_layout(P, Tm, H, K);
  const int me = static_cast<int>(rank);
  char* b = static_cast<char*>(workspace);
  // routing of the local tokens (its status word is the call's status word)
  const WsLayout R = ws_layout(T, H, I, E, K);
  char* rb = b + W.route;
  int* status = reinterpret_cast<int*>(rb + R.status);
  int32_t* idx = topk_idx_out ? topk_idx_out : reinterpret_cast<int32_t*>(rb + R.idx);
  float* w = topk_w_out ? topk_w_out : reinterpret_cast<float*>(rb + R.w);
  // completion counters: [0, P) sends, [P, 2P) returns
  unsigned* counters = reinterpret_cast<unsigned*>(b + W.counters);
  NKI_CUDA(cudaMemsetAsync(status, 0, 256, s));  // status word and router counters
  NKI_CUDA(cudaMemsetAsync(counters, 0, 256, s));
  // this step's epoch: the caller's, or this rank's device-side count + 1
  uint32_t* epoch_p = reinterpret_cast<uint32_t*>(peers.base[rank] + PL.step);
  NKI_CUDA(ep_peer_step_launch(epoch_p, epoch, s));
  if (T > 0) {
    rc = router_impl(x, router_w, router_bias, router_w_split, idx, w, T, H, E, K, rb, R, status, s);
    if (rc != NKIMOE_OK) return rc;
  }
  // the expert slots the (token, slot) pairs go to
  const int32_t* route = idx;
  if (expert_slots && T > 0) {
    int32_t* idx_v = reinterpret_cast<int32_t*>(b + W.idx_v);
    NKI_CUDA(ep_remap_launch(idx, static_cast<int>(T), static_cast<int>(K), static_cast<int>(E), expert_slots,
                             slot_counts, static_cast<int>(max_holders), static_cast<int>(P * El), idx_v, status, s));
    route = idx_v;
  }
  // (token, rank) pairs grouped by rank, tokens ascending
  mark(kStagePermute, s);
  char* db = b + W.disp;
  int32_t* offsets = reinterpret_cast<int32_t*>(db + 256);
  int32_t* dest = offsets + round256(sizeof(int32_t) * (P + 1)) / sizeof(int32_t);
  int32_t* row_token = dest + round256(sizeof(int32_t) * T * P) / sizeof(int32_t);
  int32_t* row_slot = row_token + round256(sizeof(int32_t) * T * P) / sizeof(int32_t);
  void* scratch = row_slot + round256(sizeof(int32_t) * T * P) / sizeof(int32_t);
  int32_t* slot_in = reinterpret_cast<int32_t*>(b + W.slot_in);
  int32_t* slot_out = reinterpret_cast<int32_t*>(b + W.slot_out);
  if (T > 0)
    NKI_CUDA(ep_dest_launch(route, static_cast<int>(T), static_cast<int>(K), static_cast<int>(P), static_cast<int>(El),
                            dest, s));
  NKI_CUDA(permute_launch(dest, NKIMOE_I32, static_cast<int>(T), static_cast<int>(P), static_cast<int>(P), row_token,
                          row_slot, slot_in, offsets, scratch, status, s));
  char* own = peers.base[rank];
  int32_t* recv_slots = reinterpret_cast<int32_t*>(own + PL.recv_slots);
  const float* recv_w = reinterpret_cast<const float*>(own + PL.recv_w);
  const char* recv_x = own + PL.recv_x;
  const int32_t* counts = reinterpret_cast<const int32_t*>(own + PL.counts);
  const uint32_t* disp_flag = reinterpret_cast<const uint32_t*>(own + PL.disp_flag);
  const uint32_t* res_flag = reinterpret_cast<const uint32_t*>(own + PL.res_flag);
  const long long budget = g_peer_wait_cycles.load();
  // auto: the copy-engine overlap for prefill-sized batches on 2 to 4 ranks
  // (measured at 8192 tokens per rank: 4 ranks 0.99 ms against 1.12 ms in one
  // block, 2 ranks on par); one block on more ranks, where the whole-region
  // copies of every pair of ranks outlast the expert work (8 ranks: 1.75 ms
  // against 1.55), and for decode steps (a handful of rows, where the one
  // block's few launches win).  Each rank decides for itself: every schedule
  // writes the same buffers the same way, only the order of the work differs.
  const int schedule = nkimoe_ep_peer_schedule(P, Tm);
  const bool overlapped = schedule != 0;

  if (!overlapped) {
    // ---- one block: every row (own included) through the buffers, then all
    // of this rank's experts over all P regions
    NKI_CUDA(ep_peer_local_launch(route, w, slot_in, offsets, static_cast<int>(T), static_cast<int>(K),
                                  static_cast<int>(P), static_cast<int>(El), static_cast<int>(Tm), me, false, slot_out,
                                  nullptr, nullptr, s));
    mark(kStageEpSend, s);
    NKI_CUDA(ep_peer_send_launch(static_cast<const __nv_bfloat16*>(x), route, w, row_token, row_slot, offsets,
                                 static_cast<int>(T), static_cast<int>(H), static_cast<int>(K), static_cast<int>(P),
                                 static_cast<int>(El), static_cast<int>(Tm), me, 0, static_cast<int>(P), peers, PL,
                                 counters, epoch_p, 0, s));
    mark(kStageEpWait, s);
    NKI_CUDA(ep_peer_wait_launch(disp_flag, static_cast<int>(P), epoch_p, status, budget, s));
    NKI_CUDA(ep_peer_mask_launch(recv_slots, counts, 0, static_cast<int>(P), static_cast<int>(Tm),
                                 static_cast<int>(K), s));
    const PeerCombine pc{peers, PL, static_cast<int>(P), me, static_cast<int>(Tm), 0, static_cast<int>(P), 0,
                         counters + P, epoch_p};
    rc = experts_impl(recv_x, w13_local, w2_local, recv_slots, NKIMOE_I32, recv_w, nullptr, P * Tm, H, I, El, K,
                      b + W.recv, workspace_bytes - W.recv, s, &pc, status);
    if (rc != NKIMOE_OK) return rc;
    mark(kStageEpReturnWait, s);
    NKI_CUDA(ep_peer_wait_launch(res_flag, static_cast<int>(P), epoch_p, status, budget, s));
  } else {
    // ---- overlapped: the transfers to the other ranks run on a side stream
    // of the library beside the expert GEMMs.  Schedule 1: the send and
    // return kernels store over NVLink from that stream; schedule 2: the rows
    // and sums are gathered into local staging regions on the main stream and
    // the copy engines move each destination's whole region (cudaMemcpyAsync
    // to the peer's mapped buffer, then a one-thread kernel publishes the
    // count and the flag), so the transfers take no SM time from the GEMMs.
    // The own tokens' share goes straight from x; remote regions are taken
    // in groups, nearest sources first (each source sends to its nearest
    // destination first), each group's sums returned while the next computes.
    const bool copy_engines = schedule == 2;
    int32_t* self_idx = reinterpret_cast<int32_t*>(b + W.self_idx);
    float* self_w = reinterpret_cast<float*>(b + W.self_w);
    NKI_CUDA(ep_peer_local_launch(route, w, slot_in, offsets, static_cast<int>(T), static_cast<int>(K),
                                  static_cast<int>(P), static_cast<int>(El), static_cast<int>(Tm), me, true, slot_out,
                                  self_idx, self_w, s));
    int dev = 0;
    NKI_CUDA(cudaGetDevice(&dev));
    NKI_REQUIRE(dev >= 0 && dev < kEpMaxDevices, NKIMOE_ERR_UNSUPPORTED, "device %d", dev);
    std::lock_guard<std::mutex> lock(g_ep_mu[dev]);
    EpSideStream& es = g_ep[dev];
    rc = ep_side_init(es);
    if (rc != NKIMOE_OK) return rc;
    const int side_ctas = g_ep_side_ctas.load() > 0 ? g_ep_side_ctas.load() : device_sm_count();
    long long groups = g_ep_groups.load() > 0 ? g_ep_groups.load() : std::min<long long>(P - 1, 2);
    groups = std::min<long long>(groups, P - 1);  // 0 for a single rank: no remote regions
    __nv_bfloat16* stage_x = reinterpret_cast<__nv_bfloat16*>(b + W.stage_x);
    int32_t* stage_slots = reinterpret_cast<int32_t*>(b + W.stage_slots);
    float* stage_w = reinterpret_cast<float*>(b + W.stage_w);
    int32_t* stage_counts = reinterpret_cast<int32_t*>(b + W.stage_counts);
    __nv_bfloat16* ret_stage = reinterpret_cast<__nv_bfloat16*>(b + W.ret_stage);
    const size_t region_x = sizeof(uint16_t) * Tm * H, region_k = sizeof(int32_t) * Tm * K;
    if (copy_engines)
      NKI_CUDA(ep_peer_stage_launch(static_cast<const __nv_bfloat16*>(x), route, w, row_token, row_slot, offsets,
                                    static_cast<int>(T), static_cast<int>(H), static_cast<int>(K), static_cast<int>(P),
                                    static_cast<int>(El), static_cast<int>(Tm), me, stage_x, stage_slots, stage_w,
                                    stage_counts, s));
    mark(kStageEpSend, s);
    NKI_CUDA(cudaEventRecord(es.fork, s));
    NKI_CUDA(cudaStreamWaitEvent(es.side, es.fork, 0));
    for (long long q = 1; q < P; ++q) {  // one destination after another, nearest first
      const int d = static_cast<int>((rank + q) % P);
      if (copy_engines) {
        char* pd = peers.base[d];
        NKI_CUDA(cudaMemcpyAsync(pd + PL.recv_x + q * region_x, reinterpret_cast<char*>(stage_x) + d * region_x,
                                 region_x, cudaMemcpyDeviceToDevice, es.side));
        NKI_CUDA(cudaMemcpyAsync(pd + PL.recv_slots + q * region_k,
                                 reinterpret_cast<char*>(stage_slots) + d * region_k, region_k,
                                 cudaMemcpyDeviceToDevice, es.side));
        NKI_CUDA(cudaMemcpyAsync(pd + PL.recv_w + q * region_k, reinterpret_cast<char*>(stage_w) + d * region_k,
                                 region_k, cudaMemcpyDeviceToDevice, es.side));
        NKI_CUDA(ep_peer_publish_launch(reinterpret_cast<int32_t*>(pd + PL.counts) + q, stage_counts + d,
                                        reinterpret_cast<uint32_t*>(pd + PL.disp_flag) + q, epoch_p, es.side));
      } else {
        NKI_CUDA(ep_peer_send_launch(static_cast<const __nv_bfloat16*>(x), route, w, row_token, row_slot, offsets,
                                     static_cast<int>(T), static_cast<int>(H), static_cast<int>(K),
                                     static_cast<int>(P), static_cast<int>(El), static_cast<int>(Tm), me, d, 1, peers,
                                     PL, counters + q, epoch_p, side_ctas, es.side));
      }
    }
    // own tokens: prep and the first half of the experts before the remote
    // rows are needed, the second half after them (covering the last returns)
    char* sb = b + W.recv;
    const ExpertsRun self = experts_run(x, w13_local, w2_local, self_idx, NKIMOE_I32, self_w, T, H, I, El, K, sb,
                                        status);
    const long long split = (T * K > 48 * El * P && El >= 2) ? El / 2 : El;
    rc = experts_prep(self, s, false, false);
    if (rc == NKIMOE_OK) rc = experts_gemms(self, 0, split, s, false);
    if (rc != NKIMOE_OK) return rc;
    mark(kStageEpWait, s);
    char* gb = sb + round256(ws_layout(T, H, I, El, K).total);
    for (long long g = 0; g < groups; ++g) {
      const long long q0 = group_q0(P, groups, g), nq = group_q0(P, groups, g + 1) - q0;
      NKI_CUDA(ep_peer_wait_launch(disp_flag + q0, static_cast<int>(nq), epoch_p, status, budget, s));
      NKI_CUDA(ep_peer_mask_launch(recv_slots + q0 * Tm * K, counts, static_cast<int>(q0), static_cast<int>(nq),
                                   static_cast<int>(Tm), static_cast<int>(K), s));
      const ExpertsRun grp = experts_run(recv_x + q0 * Tm * H * sizeof(uint16_t), w13_local, w2_local,
                                         recv_slots + q0 * Tm * K, NKIMOE_I32, recv_w + q0 * Tm * K, nq * Tm, H, I,
                                         El, K, gb, status);
      rc = experts_prep(grp, s, false, false);
      if (rc == NKIMOE_OK) rc = experts_gemms(grp, 0, El, s, false);
      if (rc != NKIMOE_OK) return rc;
      if (copy_engines) {
        // the group's sums into the local return regions, then each region
        // copied to its source from the side stream
        NKI_CUDA(ep_peer_combine_launch(reinterpret_cast<const __nv_bfloat16*>(gb + grp.L.xy),
                                        reinterpret_cast<const int32_t*>(gb + grp.L.slot_row), static_cast<int>(q0),
                                        static_cast<int>(nq), static_cast<int>(K), static_cast<int>(H),
                                        static_cast<int>(Tm), me, peers, PL, static_cast<int>(P), nullptr, epoch_p, 0,
                                        s, ret_stage));
        NKI_CUDA(cudaEventRecord(es.group[g], s));
        NKI_CUDA(cudaStreamWaitEvent(es.side, es.group[g], 0));
        for (long long q = q0; q < q0 + nq; ++q) {
          char* ps = peers.base[(rank - q + P) % P];
          NKI_CUDA(cudaMemcpyAsync(ps + PL.ret_y + q * region_x, reinterpret_cast<char*>(ret_stage) + q * region_x,
                                   region_x, cudaMemcpyDeviceToDevice, es.side));
          NKI_CUDA(ep_peer_publish_launch(nullptr, nullptr, reinterpret_cast<uint32_t*>(ps + PL.res_flag) + q,
                                          epoch_p, es.side));
        }
      } else {
        // the group's sums go back to their sources from the side stream
        NKI_CUDA(cudaEventRecord(es.group[g], s));
        NKI_CUDA(cudaStreamWaitEvent(es.side, es.group[g], 0));
        const PeerCombine pc{peers, PL, static_cast<int>(P), me, static_cast<int>(Tm), static_cast<int>(q0),
                             static_cast<int>(nq), side_ctas, counters + P + g, epoch_p};
        rc = experts_finish(grp, nullptr, &pc, nullptr, es.side, false);
        if (rc != NKIMOE_OK) return rc;
      }
      gb += round256(ws_layout(nq * Tm, H, I, El, K).total);
    }
    mark(kStageEpReturnWait, s);
    rc = experts_gemms(self, split, El, s, false);
    if (rc == NKIMOE_OK) rc = experts_finish(self, own + PL.ret_y, nullptr, nullptr, s, false);
    if (rc != NKIMOE_OK) return rc;
    if (P > 1) NKI_CUDA(ep_peer_wait_launch(res_flag + 1, static_cast<int>(P - 1), epoch_p, status, budget, s));
    // the side stream's work belongs to this call
    NKI_CUDA(cudaEventRecord(es.join, es.side));
    NKI_CUDA(cudaStreamWaitEvent(s, es.join, 0));
  }
  mark(kStageEpSum, s);
  if (T > 0)
    NKI_CUDA(combine_launch(reinterpret_cast<const __nv_bfloat16*>(own + PL.ret_y), slot_out, nullptr,
                            static_cast<__nv_bfloat16*>(out), static_cast<int>(T), static_cast<int>(P),
                            static_cast<int>(H), s));
  mark(kStageEpEnd, s);
  return NKIMOE_OK;
}

int nkimoe_ep_peer_forward(const void* x, const float* router_w, const float* router_bias, const void* router_w_split,
                           const void* w13_local, const void* w2_local, void* out, int32_t* topk_idx_out,
                           float* topk_w_out, int64_t T, int64_t H, int64_t I,
                           int64_t E, int64_t K, int64_t num_ranks, int64_t rank, int64_t max_tokens,
                           void* const* peer_buffers, uint32_t epoch, void* workspace, size_t workspace_bytes,
                           void* stream) {
  NKI_REQUIRE(num_ranks >= 1 && E % num_ranks == 0, NKIMOE_ERR_UNSUPPORTED, "ep peer: ranks must divide the experts");
  return ep_peer_forward_impl(x, router_w, router_bias, router_w_split, w13_local, w2_local, out, topk_idx_out,
                              topk_w_out, T, H, I, E, K, num_ranks, rank, max_tokens, peer_buffers, epoch, workspace,
                              workspace_bytes, stream, E / num_ranks, nullptr, nullptr, 0);
}

int nkimoe_ep_peer_forward_mapped(const void* x, const float* router_w, const float* router_bias,
                                  const void* router_w_split, const void* w13_local, const void* w2_local, void* out,
                                  int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I,
                                  int64_t E, int64_t K, int64_t num_ranks, int64_t rank, int64_t max_tokens,
                                  void* const* peer_buffers, uint32_t epoch, void* workspace,
                                  size_t workspace_bytes, void* stream, int64_t local_slots,
                                  const int32_t* expert_slots, const int32_t* slot_counts, int64_t max_holders) {
  NKI_REQUIRE(expert_slots && slot_counts, NKIMOE_ERR_INVALID_ARG, "ep peer: null expert slot map");
  return ep_peer_forward_impl(x, router_w, router_bias, router_w_split, w13_local, w2_local, out, topk_idx_out,
                              topk_w_out, T, H, I, E, K, num_ranks, rank, max_tokens, peer_buffers, epoch, workspace,
                              workspace_bytes, stream, local_slots, expert_slots, slot_counts, max_holders);
}

int nkimoe_combine(const void* y, const int32_t* slot_row, const float* slot_weight, void* out, int64_t T, int64_t K,
                   int64_t H, void* stream) {
  NKI_REQUIRE(T >= 0 && K > 0 && H > 0 && H % 8 == 0, NKIMOE_ERR_INVALID_ARG, "combine: bad shape");
  NKI_REQUIRE(T * (H / 8) < (1LL << 31) && T * K < (1LL << 31), NKIMOE_ERR_UNSUPPORTED, "combine: T too large");
  if (T == 0) return NKIMOE_OK;
  NKI_REQUIRE(y && slot_row && out && aligned16(y) && aligned16(out), NKIMOE_ERR_INVALID_ARG,
              "null or misaligned pointer");
  NKI_CUDA(combine_launch(static_cast<const __nv_bfloat16*>(y), slot_row, slot_weight, static_cast<__nv_bfloat16*>(out),
                          static_cast<int>(T), static_cast<int>(K), static_cast<int>(H), as_stream(stream)));
  return NKIMOE_OK;
}

}  // extern "C"
