// K2: router of the sparse-MoE block (nki_moe_integrated.py:436-443):
//   logits = x . Wr^T in fp32 (router dtype fp32, qwen_with_nki.py:276),
//   p = softmax(logits), (w, idx) = topk(p, K) descending, w /= sum(w).
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "kernels.h"
#include "permute_small.cuh"

namespace nkimoe {

namespace {

// 64 tokens x 64 experts per CTA, 256 threads, 4x4 outputs per thread,
// K staged through shared memory 32 at a time; each output is one fp32 FMA
// chain in ascending k (deterministic, no TF32).
constexpr int RT = 64, RE = 64, RK = 32;

__global__ void __launch_bounds__(256) router_logits_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const float* __restrict__ wr,
                                                            const float* __restrict__ bias, float* __restrict__ logits,
                                                            int T, int H, int E) {
  __shared__ __align__(16) float xs[RK][RT + 4];
  __shared__ __align__(16) float ws[RK][RE + 4];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * RT, e0 = blockIdx.y * RE;
  const int ty = tid >> 4, tx = tid & 15;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < H; k0 += RK) {
    {  // x tile: 64 tokens x 32 k (bf16), one 8-element chunk per thread
      const int r = tid >> 2, c = (tid & 3) * 8;
      float v[8] = {};
      if (t0 + r < T) {
        uint4 u = *reinterpret_cast<const uint4*>(x + static_cast<long long>(t0 + r) * H + k0 + c);
        float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), cc = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = cc.x; v[5] = cc.y; v[6] = d.x; v[7] = d.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) xs[c + j][r] = v[j];
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // w tile: 64 experts x 32 k (fp32)
      const int idx = tid + i * 256;
      const int r = idx >> 3, c = (idx & 7) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + r < E) v = *reinterpret_cast<const float4*>(wr + static_cast<long long>(e0 + r) * H + k0 + c);
      ws[c + 0][r] = v.x;
      ws[c + 1][r] = v.y;
      ws[c + 2][r] = v.z;
      ws[c + 3][r] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < RK; ++k) {
      const float4 a = *reinterpret_cast<const float4*>(&xs[k][ty * 4]);
      const float4 b = *reinterpret_cast<const float4*>(&ws[k][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + ty * 4 + i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = e0 + tx * 4 + j;
      if (e < E) logits[static_cast<long long>(t) * E + e] = acc[i][j] + (bias ? bias[e] : 0.f);
    }
  }
}

// Split-K variant for few tokens: a CTA computes 16 tokens x 128 experts over
// one K span and writes fp32 partial sums [split][T][E]; the top-k kernel adds
// the splits in ascending order (deterministic).  Each output of a split is
// one FMA chain in ascending k.
constexpr int ST = 16, SE = 128, SK = 32;

__global__ void __launch_bounds__(256) router_splitk_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const float* __restrict__ wr,
                                                            float* __restrict__ partial, int T, int H, int E,
                                                            int kspan) {
  __shared__ __align__(16) float xs[SK][ST];
  __shared__ __align__(16) float ws[SK][SE + 4];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * ST, e0 = blockIdx.y * SE;
  const int kb = blockIdx.z * kspan, ke = min(H, kb + kspan);
  const int tt = tid >> 4, eg = (tid & 15) * 8;
  float acc[8] = {};
  for (int k0 = kb; k0 < ke; k0 += SK) {
    if (tid < 64) {  // x: 16 tokens x 32 k, 8 bf16 per thread
      const int r = tid >> 2, c = (tid & 3) * 8;
      float v[8] = {};
      if (t0 + r < T) {
        uint4 u = *reinterpret_cast<const uint4*>(x + static_cast<long long>(t0 + r) * H + k0 + c);
        float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), cc = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
        v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = cc.x; v[5] = cc.y; v[6] = d.x; v[7] = d.y;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) xs[c + j][r] = v[j];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // w: 128 experts x 32 k fp32
      const int idx = tid + i * 256;
      const int r = idx >> 3, c = (idx & 7) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e0 + r < E) v = *reinterpret_cast<const float4*>(wr + static_cast<long long>(e0 + r) * H + k0 + c);
      ws[c + 0][r] = v.x;
      ws[c + 1][r] = v.y;
      ws[c + 2][r] = v.z;
      ws[c + 3][r] = v.w;
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < SK; ++k) {
      const float a = xs[k][tt];
      const float4 b0 = *reinterpret_cast<const float4*>(&ws[k][eg]);
      const float4 b1 = *reinterpret_cast<const float4*>(&ws[k][eg + 4]);
      acc[0] = fmaf(a, b0.x, acc[0]);
      acc[1] = fmaf(a, b0.y, acc[1]);
      acc[2] = fmaf(a, b0.z, acc[2]);
      acc[3] = fmaf(a, b0.w, acc[3]);
      acc[4] = fmaf(a, b1.x, acc[4]);
      acc[5] = fmaf(a, b1.y, acc[5]);
      acc[6] = fmaf(a, b1.z, acc[6]);
      acc[7] = fmaf(a, b1.w, acc[7]);
    }
    __syncthreads();
  }
  const int t = t0 + tt;
  if (t < T) {
    float* dst = partial + (static_cast<long long>(blockIdx.z) * T + t) * E;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (e0 + eg + j < E) dst[e0 + eg + j] = acc[j];
  }
}

__global__ void router_split_kernel(const float* __restrict__ wr, __nv_bfloat16* __restrict__ out, int E, int H) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(E) * H) return;
  const int e = static_cast<int>(i / H), h = static_cast<int>(i % H);
  const float w = wr[i];
  const __nv_bfloat16 hi = __float2bfloat16_rn(w);
  const float r1 = w - __bfloat162float(hi);
  const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  const float r2 = r1 - __bfloat162float(mid);
  const __nv_bfloat16 lo = __float2bfloat16_rn(r2);
  const long long plane = static_cast<long long>(E) * H;
  out[static_cast<long long>(e) * H + h] = hi;
  out[plane + static_cast<long long>(e) * H + h] = mid;
  out[2 * plane + static_cast<long long>(e) * H + h] = lo;
}

// Order-preserving map of a float to u32 (a > b  <=>  key(a) > key(b)).
__device__ __forceinline__ uint32_t order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if (u == 0x80000000u) u = 0u;  // -0 == +0 (a tie, broken by id)
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Softmax -> top-k -> renormalise for one token held by a warp: lane l holds
// the logits of experts l, l+32, ... (v[j] = expert l + 32 j, -inf past E).
// Selection is by logit, ties to the lower id; p = exp(v - max) / sum.
// Each lane sorts its VPT values (descending, ties by id); a round takes the
// warp maximum of the lane heads (redux.sync on an order-preserving key) and
// the lowest id holding it (a second redux), and the winning lane pops its
// head.
template <int VPT>
__device__ __forceinline__ void topk_select_warp(const float (&v)[VPT], int E, int K, int lane,
                                                 int32_t* __restrict__ idx_row, float* __restrict__ w_row) {
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < VPT; ++j) m = fmaxf(m, v[j]);
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = lane + 32 * j;
    if (e < E) s += expf(v[j] - m);
  }
  s = warp_sum(s);
  // this lane's candidates, sorted descending (stable: equal values keep the
  // lower id first); past-E slots carry key 0 (below every real logit)
  uint32_t key[VPT];
  int id[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    id[j] = lane + 32 * j;
    key[j] = id[j] < E ? order_key(v[j]) : 0u;
  }
#pragma unroll
  for (int i = 1; i < VPT; ++i) {
#pragma unroll
    for (int j = i; j > 0; --j) {
      const bool sw = key[j] > key[j - 1];
      const uint32_t tk = sw ? key[j - 1] : key[j];
      const int ti = sw ? id[j - 1] : id[j];
      key[j - 1] = sw ? key[j] : key[j - 1];
      id[j - 1] = sw ? id[j] : id[j - 1];
      key[j] = tk;
      id[j] = ti;
    }
  }
  int my_idx = 0;
  float my_p = 0.f;
  for (int r = 0; r < K; ++r) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, key[0]);
    const int win = static_cast<int>(
        __reduce_min_sync(0xffffffffu, key[0] == best ? static_cast<uint32_t>(id[0]) : 0xffffffffu));
    if (lane == r) {
      my_idx = win;
      const uint32_t bits = (best & 0x80000000u) ? (best & 0x7fffffffu) : ~best;
      my_p = expf(__uint_as_float(bits) - m) / s;
    }
    if (id[0] == win) {  // the winner pops its head
#pragma unroll
      for (int j = 0; j + 1 < VPT; ++j) {
        key[j] = key[j + 1];
        id[j] = id[j + 1];
      }
      key[VPT - 1] = 0u;
      id[VPT - 1] = 0x7fffffff;
    }
  }
  float tot = warp_sum(lane < K ? my_p : 0.f);
  if (lane < K) {
    idx_row[lane] = my_idx;
    w_row[lane] = my_p / tot;
  }
}

// One warp per token; lane l holds experts l, l+32, ... (VPT of them).
// The logits of token t are sum_{s < splits} partial[s][t][:] (+ bias), added
// in ascending s; with splits = 1 and no bias they are read as they are.
template <int VPT>
__global__ void __launch_bounds__(256) topk_softmax_kernel(const float* __restrict__ partial, int splits,
                                                           const float* __restrict__ bias,
                                                           float* __restrict__ logits_out, int T, int E, int K,
                                                           int32_t* __restrict__ idx_out, float* __restrict__ w_out) {
  const int lane = threadIdx.x & 31;
  const long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  // every split's partial is loaded before any is added (one round trip, not
  // one per split); the sum keeps ascending split order
  constexpr int kMaxSplits = 8;
  float pv[VPT][kMaxSplits];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = lane + 32 * j;
#pragma unroll
    for (int sp = 0; sp < kMaxSplits; ++sp)
      pv[j][sp] = (e < E && sp < splits) ? partial[(static_cast<long long>(sp) * T + t) * E + e] : 0.f;
  }
  float v[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int e = lane + 32 * j;
    if (e < E) {
      float acc = pv[j][0];
#pragma unroll
      for (int sp = 1; sp < kMaxSplits; ++sp)
        if (sp < splits) acc += pv[j][sp];
      if (bias) acc += bias[e];
      if (logits_out) logits_out[t * E + e] = acc;
      v[j] = acc;
    } else {
      v[j] = -INFINITY;
    }
  }
  topk_select_warp<VPT>(v, E, K, lane, idx_out + t * K, w_out + t * K);
}

// Router logits of a prefill batch in one tensor-core kernel, with an
// optional RMSNorm of the rows in front of it.  CTA = 128 rows x one half of
// the experts (two CTAs per row block, so a batch fills twice as many SMs);
// the fp32 router weights are three exact bf16 planes (hi, mid, lo;
// router_split_kernel) and each plane has its own TMEM accumulator (3 x 64
// columns).  The MMAs are
// those of the router GEMM (M128 K16, K ascending, one accumulator per plane;
// N = 64 experts here, 128 there: each logit is the same sum) and the epilogue adds the planes as topk_softmax_kernel adds split
// partials, ((hi + mid) + lo) + bias, so the logits it writes give the same
// top-k bit for bit; the top-k itself stays a separate kernel (spread over the
// whole GPU it is several times faster than in these 64-128 CTAs' epilogues).
// With the norm, the A operand of every 64-wide K block is the row block
// normalised by the CTA itself (rmsnorm_kernel's arithmetic: the lane-chunk
// fp32 sum of squares of a warp per row, (x * rsqrt) * w rounded to bf16),
// written to shared memory in the TMA 128-byte swizzle and to x_out for the
// expert gather, so the normalised rows are produced once and consumed by the
// router in the same pass (the reference's fused post-attention norm,
// qwen_with_nki.py:379-382, :451-452).
//   warps 0-3: row workers (norm, A blocks), then the epilogue (TMEM lanes
//              32 w .. 32 w + 31 = rows; fp32 logits rows to global memory)
//   warp 4:    TMA producer (router planes; the x block without the norm)
//   warp 5:    MMA issuer, TMEM owner
constexpr int kRtRows = 128, kRtBK = 64, kRtE = 128, kRtThreads = 192, kRtMaxStages = 5;
constexpr uint32_t kRtABytes = kRtRows * kRtBK * 2;      // 16 KB
// EH experts per CTA (64: two CTAs per row block, the default; 128: one)
template <int EH>
struct RtShape {
  static constexpr int kStages = EH == 128 ? 3 : 5;
  static constexpr uint32_t kBBytes = 3 * EH * kRtBK * 2;  // three planes of the CTA's experts
  static constexpr uint32_t kStageBytes = kRtABytes + kBBytes;
  static constexpr uint32_t kTmemCols = EH == 128 ? 512 : 256;
};

struct RtCtl {
  uint64_t full[kRtMaxStages], empty[kRtMaxStages], afull[kRtMaxStages];
  uint64_t acc_full, drain;
  uint32_t tmem_base;
  int abort_flag;
  float rinv[kRtRows];
};

__device__ __forceinline__ float rt_weight(const void* w, int w_dtype, int k) {
  return w_dtype == 0 ? static_cast<const float*>(w)[k] : __bfloat162float(static_cast<const __nv_bfloat16*>(w)[k]);
}

template <bool kNorm, int EH>
__global__ void __launch_bounds__(kRtThreads, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                     const __nv_bfloat16* __restrict__ h, const void* __restrict__ norm_w, int norm_w_dtype,
                     float eps, __nv_bfloat16* __restrict__ x_out, const float* __restrict__ bias,
                     float* __restrict__ logits_out, int T, int H, int* status) {
  extern __shared__ uint8_t rt_smem_raw[];
  __shared__ RtCtl ctl;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(rt_smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  using S = RtShape<EH>;
  const long long row0 = static_cast<long long>(blockIdx.x / (kRtE / EH)) * kRtRows;
  const int eh = static_cast<int>(blockIdx.x % (kRtE / EH));  // experts [EH eh, EH eh + EH)
  const int kblocks = H / kRtBK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&ctl.full[s], 1);
      mbar_init(&ctl.empty[s], 1);
      mbar_init(&ctl.afull[s], 4 * 32);
    }
    mbar_init(&ctl.acc_full, 1);
    mbar_init(&ctl.drain, 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&tmap_w);
    if (!kNorm) prefetch_tmap(&tmap_x);
  }
  if (warp == 5) tmem_alloc(&ctl.tmem_base, S::kTmemCols);
  if (kNorm && warp < 4) {
    // sum of squares of each row as rmsnorm_kernel forms it: lane l adds the
    // squares of chunks l + 32 i (8 bf16 each) in order, then a butterfly
    for (int rl = warp; rl < kRtRows; rl += 4) {
      const long long row = row0 + rl;
      float ss = 0.f;
      if (row < T) {
        const __nv_bfloat16* xr = h + row * H;
        float v[8][8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = lane + i * 32;
          if (c < (H >> 3)) {
            const uint4 u = *reinterpret_cast<const uint4*>(xr + c * 8);
            const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), cc = unpack_bf16x2(u.z),
                         d = unpack_bf16x2(u.w);
            v[i][0] = a.x; v[i][1] = a.y; v[i][2] = b.x; v[i][3] = b.y;
            v[i][4] = cc.x; v[i][5] = cc.y; v[i][6] = d.x; v[i][7] = d.y;
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = lane + i * 32;
          if (c < (H >> 3)) {
#pragma unroll
            for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
          }
        }
      }
      ss = warp_sum(ss);
      if (lane == 0) ctl.rinv[rl] = rsqrtf(ss / static_cast<float>(H) + eps);
    }
  }
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0, issued = 0, last = 0;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&ctl.empty[stage], phase ^ 1u, &ctl.abort_flag, status)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + stage * S::kStageBytes;
        mbar_arrive_expect_tx(&ctl.full[stage], kNorm ? S::kBBytes : S::kStageBytes);
        if (!kNorm) tma_load_2d(st, &tmap_x, &ctl.full[stage], kb * kRtBK, static_cast<int>(row0));
#pragma unroll
        for (int p = 0; p < 3; ++p)
          tma_load_2d(st + kRtABytes + p * (EH * kRtBK * 2), &tmap_w, &ctl.full[stage], kb * kRtBK,
                      p * kRtE + eh * EH);
        issued |= 1u << stage;
        last = (last & ~(1u << stage)) | (phase << stage);
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok)  // let copies in flight land before the CTA exits
        for (int s = 0; s < S::kStages; ++s)
          if ((issued >> s) & 1u) {
            const long long t0 = clock64();
            while (!mbar_try_wait(&ctl.full[s], (last >> s) & 1u))
              if (clock64() - t0 > kWaitBudgetCycles / 8) break;
          }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kRtRows, EH);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, any = false;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(&ctl.full[stage], phase, &ctl.abort_flag, status) ||
            (kNorm && !mbar_wait(&ctl.afull[stage], phase, &ctl.abort_flag, status))) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        uint8_t* st = smem + stage * S::kStageBytes;
        const uint64_t da = umma_desc_sw128(smem_u32(st));
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const uint64_t db = umma_desc_sw128(smem_u32(st + kRtABytes + p * (EH * kRtBK * 2)));
#pragma unroll
          for (int kk = 0; kk < kRtBK / 16; ++kk)
            umma_bf16(tmem_base + p * EH, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&ctl.empty[stage]);
        any = true;
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok) {
        umma_commit(&ctl.acc_full);
      } else if (any) {  // wait for issued MMAs before TMEM is released
        umma_commit(&ctl.drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(&ctl.drain, 0))
          if (clock64() - t0 > kWaitBudgetCycles / 8) break;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ row workers
    bool ok = true;
    if (kNorm) {
      // A block kb: thread t fills 16-byte chunk t % 8 of rows t / 8 + 16 i
      const int c = threadIdx.x & 7;
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = 0; kb < kblocks && ok; ++kb) {
        bool got = true;
        if (lane == 0) got = mbar_wait(&ctl.empty[stage], phase ^ 1u, &ctl.abort_flag, status);
        if (__shfl_sync(0xffffffffu, got ? 1 : 0, 0) == 0) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + stage * S::kStageBytes;
        const int k0 = kb * kRtBK + c * 8;
        float wv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) wv[j] = rt_weight(norm_w, norm_w_dtype, k0 + j);
        uint4 in[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rl = (threadIdx.x >> 3) + 16 * i;
          const long long row = row0 + rl;
          in[i] = row < T ? *reinterpret_cast<const uint4*>(h + row * H + k0) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rl = (threadIdx.x >> 3) + 16 * i;
          const long long row = row0 + rl;
          uint4 o = make_uint4(0, 0, 0, 0);
          if (row < T) {
            const float r = ctl.rinv[rl];
            const float2 a = unpack_bf16x2(in[i].x), b = unpack_bf16x2(in[i].y), cc = unpack_bf16x2(in[i].z),
                         d = unpack_bf16x2(in[i].w);
            o.x = pack_bf16x2(a.x * r * wv[0], a.y * r * wv[1]);
            o.y = pack_bf16x2(b.x * r * wv[2], b.y * r * wv[3]);
            o.z = pack_bf16x2(cc.x * r * wv[4], cc.y * r * wv[5]);
            o.w = pack_bf16x2(d.x * r * wv[6], d.y * r * wv[7]);
            if (eh == 0) *reinterpret_cast<uint4*>(x_out + row * H + k0) = o;
          }
          *reinterpret_cast<uint4*>(sa + rl * 128 + ((c ^ (rl & 7)) << 4)) = o;
        }
        fence_proxy_async_shared();  // generic-proxy writes -> tensor-core reads
        mbar_arrive(&ctl.afull[stage]);
        if (++stage == S::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // ------------------------------------------------------------ epilogue
    bool got = ok;
    if (got && lane == 0) got = mbar_wait(&ctl.acc_full, 0, &ctl.abort_flag, status);
    got = __shfl_sync(0xffffffffu, got ? 1 : 0, 0) != 0;
    if (got) {
      tcgen05_fence_after();
      const long long row = row0 + warp * 32 + lane;
      const uint32_t tl = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < EH; c0 += 32) {
        uint32_t a[32], b[32], d[32];
        tmem_ld_32x32b_x32(tl + c0, a);
        tmem_ld_32x32b_x32(tl + EH + c0, b);
        tmem_ld_32x32b_x32(tl + 2 * EH + c0, d);
        tmem_ld_wait();
        float lg[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float acc = __uint_as_float(a[j]);
          acc += __uint_as_float(b[j]);
          acc += __uint_as_float(d[j]);
          if (bias) acc += bias[eh * EH + c0 + j];
          lg[j] = acc;
        }
        if (row < T) {
          float4* dst = reinterpret_cast<float4*>(logits_out + row * kRtE + eh * EH + c0);
#pragma unroll
          for (int q = 0; q < 8; ++q) dst[q] = make_float4(lg[4 * q], lg[4 * q + 1], lg[4 * q + 2], lg[4 * q + 3]);
        }
      }
    }
  }
  tcgen05_fence_before();
  __syncthreads();
  if (warp == 5) {
    tcgen05_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// Router + softmax + top-k for few tokens (decode), in one launch spread over
// many SMs (the work is 2*T*H*E FLOP on E*H*4 bytes of weights, so a handful
// of SMs would be compute-bound).  CTA (eb, s, g) computes fp32 partial
// logits of experts [8 eb, 8 eb + 8) -- one per warp -- for the 8 tokens of
// group g over the hidden slice s: lane (token tl, quarter kc) runs one FMA
// chain over k = k0 + 32 kc + [0, 32) of every 128-wide block of the slice,
// and the four quarters are added with a fixed butterfly.  The partials go to
// partial[s][t][e]; the last CTA of the group to finish (device-scope counter,
// no spinning) adds the slices in ascending order and selects each token's
// top-k (one warp per token).  The counters start at zero (the caller clears
// them with the status word) and are left at zero.
constexpr int kRouterTokens = 8;
constexpr int kRouterExpertsPerCta = 8;
constexpr int kRouterMaxSlices = 8;
constexpr int kRouterMaxGroups = 48;  // counters in the 256-byte status block, after 64 bytes

template <int VPT>
__global__ void __launch_bounds__(256)
    router_topk_split_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ wr,
                             const float* __restrict__ bias, float* __restrict__ logits_out, int T, int H, int E,
                             int K, int32_t* __restrict__ idx_out, float* __restrict__ w_out, float* partial,
                             int* counters, int kslice, RouterPermOut perm) {
  __shared__ int s_last;
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int eb = blockIdx.x, sl = blockIdx.y, gi = blockIdx.z;
  const int e = eb * kRouterExpertsPerCta + warp;
  const int tl = lane >> 2, kc = lane & 3;
  const long long t = static_cast<long long>(gi) * kRouterTokens + tl;
  const int kb = sl * kslice, ke = min(H, kb + kslice);
  float acc = 0.f;
  if (e < E) {
    const float* we = wr + static_cast<long long>(e) * H;
    const __nv_bfloat16* xt = x + (t < T ? t : 0) * H;
    // two 128-wide blocks per step: all of a lane's loads for them in flight
    for (int k0 = kb + 32 * kc; k0 < ke; k0 += 256) {
      const bool two = k0 + 128 < ke;
      float4 w4[2][8];
      uint4 xu[2][4];
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const int k = k0 + 128 * hb;
        const bool live = hb == 0 || two;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          w4[hb][q] = live ? *reinterpret_cast<const float4*>(we + k + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          xu[hb][q] = live ? *reinterpret_cast<const uint4*>(xt + k + 8 * q) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        if (hb == 1 && !two) break;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 a = unpack_bf16x2(xu[hb][q].x), b = unpack_bf16x2(xu[hb][q].y);
          const float2 c = unpack_bf16x2(xu[hb][q].z), d = unpack_bf16x2(xu[hb][q].w);
          const float4 w0 = w4[hb][2 * q], w1 = w4[hb][2 * q + 1];
          acc = fmaf(a.x, w0.x, acc);
          acc = fmaf(a.y, w0.y, acc);
          acc = fmaf(b.x, w0.z, acc);
          acc = fmaf(b.y, w0.w, acc);
          acc = fmaf(c.x, w1.x, acc);
          acc = fmaf(c.y, w1.y, acc);
          acc = fmaf(d.x, w1.z, acc);
          acc = fmaf(d.y, w1.w, acc);
        }
      }
    }
  }
  acc += __shfl_xor_sync(0xffffffffu, acc, 1);
  acc += __shfl_xor_sync(0xffffffffu, acc, 2);
  if (kc == 0 && e < E && t < T) __stcg(partial + (static_cast<long long>(sl) * T + t) * E + e, acc);

  // the CTA barrier orders the partial stores before thread 0's fence and count
  __syncthreads();
  const int total = gridDim.x * gridDim.y;
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(counters + gi, 1);
    s_last = (done == total - 1);
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;
  const long long tt = static_cast<long long>(gi) * kRouterTokens + warp;
  if (tt < T) {
    // every partial of the token is loaded before the first add (one L2
    // round trip), then the slices are added in ascending order
    const int nsl = static_cast<int>(gridDim.y);
    float pv[VPT][kRouterMaxSlices];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int ee = lane + 32 * j;
#pragma unroll
      for (int s2 = 0; s2 < kRouterMaxSlices; ++s2)
        pv[j][s2] = (ee < E && s2 < nsl) ? __ldcg(partial + (static_cast<long long>(s2) * T + tt) * E + ee) : 0.f;
    }
    float v[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int ee = lane + 32 * j;
      v[j] = -INFINITY;
      if (ee < E) {
        float sum = pv[j][0];
#pragma unroll
        for (int s2 = 1; s2 < kRouterMaxSlices; ++s2)
          if (s2 < nsl) sum += pv[j][s2];
        if (bias) sum += bias[ee];
        if (logits_out) logits_out[tt * E + ee] = sum;
        v[j] = sum;
      }
    }
    topk_select_warp<VPT>(v, E, K, lane, idx_out + tt * K, w_out + tt * K);
  }
  if (threadIdx.x == 0) counters[gi] = 0;
  if (perm.row_token != nullptr) {  // one token group: its permutation too
    __syncthreads();                // the group's idx / w, stored by the 8 warps above
    permute_small_cta<int32_t>(idx_out, T, K, E, perm.row_token, perm.row_slot, perm.slot_row, perm.expert_offsets,
                               w_out, perm.row_weight, perm.status);
  }
}

// Router + softmax + top-k for a decode batch of more than one token group
// (9..255 tokens), in one launch: an 8-CTA cluster takes 8 tokens; CTA c computes the fp32 logits of experts
// [c EG, (c + 1) EG) for those tokens (it reads only its 1/8 of the router
// weights), keeps them in shared memory, and after a cluster barrier warp 0
// of CTA c gathers token t0 + c's E logits from the 8 CTAs (distributed
// shared memory) and selects its top-k.  A logit is one fp32 FMA chain per
// lane over k = 4 lane + 128 i + j, then a butterfly sum over the lanes.
constexpr int kRouterCluster = 8;

template <int EG>
__global__ void __cluster_dims__(kRouterCluster, 1, 1) __launch_bounds__(256)
    router_topk_cluster_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ wr,
                               const float* __restrict__ bias, float* __restrict__ logits_out, int T, int H, int E,
                               int K, int32_t* __restrict__ idx_out, float* __restrict__ w_out, int* counter,
                               RouterPermOut perm) {
  extern __shared__ __align__(16) __nv_bfloat16 xs[];  // [8][H]: the cluster's token rows
  __shared__ float lg[kRouterCluster][EG];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const long long t0 = static_cast<long long>(blockIdx.x / kRouterCluster) * kRouterCluster;
  // stage the 8 token rows: every thread's loads are issued before its stores
  const int hc = H >> 3;  // 16-byte chunks per row
  for (int i0 = threadIdx.x; i0 < kRouterCluster * hc; i0 += 8 * blockDim.x) {
    uint4 u[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = i0 + q * blockDim.x, r = i / hc, c = i - r * hc;
      u[q] = make_uint4(0u, 0u, 0u, 0u);
      if (i < kRouterCluster * hc && t0 + r < T) u[q] = reinterpret_cast<const uint4*>(x + (t0 + r) * H)[c];
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = i0 + q * blockDim.x, r = i / hc, c = i - r * hc;
      if (i < kRouterCluster * hc) reinterpret_cast<uint4*>(xs + static_cast<long long>(r) * H)[c] = u[q];
    }
  }
  __syncthreads();
  for (int el = warp; el < EG; el += 8) {
    const int e = static_cast<int>(rank) * EG + el;
    float acc[kRouterCluster] = {};
    if (e < E) {
      const float* we = wr + static_cast<long long>(e) * H;
      for (int k0 = 4 * lane; k0 < H; k0 += 16 * 128) {
        float4 w4[16];  // 16 weight loads in flight per lane
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int k = k0 + 128 * q;
          w4[q] = k < H ? *reinterpret_cast<const float4*>(we + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int k = k0 + 128 * q;
          if (k >= H) break;
#pragma unroll
          for (int t = 0; t < kRouterCluster; ++t) {
            const uint2 u = *reinterpret_cast<const uint2*>(xs + static_cast<long long>(t) * H + k);
            const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
            acc[t] = fmaf(a.x, w4[q].x, acc[t]);
            acc[t] = fmaf(a.y, w4[q].y, acc[t]);
            acc[t] = fmaf(b.x, w4[q].z, acc[t]);
            acc[t] = fmaf(b.y, w4[q].w, acc[t]);
          }
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kRouterCluster; ++t) {
      const float sum = warp_sum(acc[t]);
      if (lane == 0) lg[t][el] = sum;
    }
  }
  cluster_sync();  // every CTA's logits written and visible to the cluster
  const long long t = t0 + rank;
  if (warp == 0 && t < T) {
    constexpr int VPT = (kRouterCluster * EG + 31) / 32;
    float v[VPT];
    const uint32_t lg_local = smem_u32(&lg[rank][0]);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int e = lane + 32 * j;
      v[j] = -INFINITY;
      if (e < E) {
        const uint32_t src = mapa_shared(lg_local + static_cast<uint32_t>(e % EG) * 4u, static_cast<uint32_t>(e / EG));
        float val;
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(val) : "r"(src) : "memory");
        if (bias) val += bias[e];
        if (logits_out) logits_out[t * E + e] = val;
        v[j] = val;
      }
    }
    topk_select_warp<VPT>(v, E, K, lane, idx_out + t * K, w_out + t * K);
  }
  cluster_sync();  // no CTA leaves while another still reads its logits
  if (perm.row_token != nullptr) {
    // the last CTA of the grid to finish (device-scope counter, no spinning)
    // holds every token's routing: it writes the permutation
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
      __threadfence();
      s_last = atomicAdd(counter, 1) == static_cast<int>(gridDim.x) - 1;
      if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    if (threadIdx.x == 0) *counter = 0;
    permute_small_cta<int32_t>(idx_out, T, K, E, perm.row_token, perm.row_slot, perm.slot_row, perm.expert_offsets,
                               w_out, perm.row_weight, perm.status);
  }
}

}  // namespace

cudaError_t router_logits_simt_launch(const __nv_bfloat16* x, const float* wr, const float* bias, float* logits,
                                      int tokens, int hidden, int experts, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (hidden % RK) return cudaErrorInvalidValue;
  dim3 grid((tokens + RT - 1) / RT, (experts + RE - 1) / RE);
  router_logits_kernel<<<grid, 256, 0, s>>>(x, wr, bias, logits, tokens, hidden, experts);
  return cudaGetLastError();
}

cudaError_t router_split_launch(const float* wr, __nv_bfloat16* wsplit, int experts, int hidden, cudaStream_t s) {
  const long long n = static_cast<long long>(experts) * hidden;
  router_split_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(wr, wsplit, experts, hidden);
  return cudaGetLastError();
}

cudaError_t router_splitk_launch(const __nv_bfloat16* x, const float* wr, float* partial, int tokens, int hidden,
                                 int experts, int splits, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (hidden % SK || splits < 1) return cudaErrorInvalidValue;
  const int kspan = ((hidden / splits + SK - 1) / SK) * SK;
  dim3 grid((tokens + ST - 1) / ST, (experts + SE - 1) / SE, (hidden + kspan - 1) / kspan);
  router_splitk_kernel<<<grid, 256, 0, s>>>(x, wr, partial, tokens, hidden, experts, kspan);
  return cudaGetLastError();
}

int router_splits_for(int tokens, int hidden, int experts) {
  // about a quarter of the SMs busy and at most 8 partial sums per logit: the
  // router reads only E*H*4 bytes, latency matters more than bandwidth
  const long long tiles = static_cast<long long>((tokens + ST - 1) / ST) * ((experts + SE - 1) / SE);
  long long sp = (device_sm_count() / 4 + tiles - 1) / tiles;
  sp = std::max<long long>(1, std::min<long long>({sp, 8LL, static_cast<long long>(hidden / SK)}));
  const int kspan = static_cast<int>(((hidden / sp + SK - 1) / SK) * SK);
  return (hidden + kspan - 1) / kspan;  // the number of splits actually launched
}

bool router_topk_fused_supported(int hidden, int experts, int top_k) {
  return experts >= 1 && experts <= 256 && hidden % 128 == 0 && top_k >= 1 && top_k <= 32 && top_k <= experts;
}

int router_topk_slices(int tokens, int hidden, int experts) {
  // as many slices as fit one wave of resident CTAs (3 per SM at 256 threads x
  // up to 80 registers): a second wave would add a whole round of load latency
  const int groups = (tokens + kRouterTokens - 1) / kRouterTokens;
  const int eblocks = (experts + kRouterExpertsPerCta - 1) / kRouterExpertsPerCta;
  const int wave = 3 * device_sm_count();
  const int sl = std::max(1, std::min(kRouterMaxSlices, wave / std::max(1, groups * eblocks)));
  const int blocks = hidden / 128;
  const int per = (blocks + sl - 1) / sl;  // 128-wide blocks per slice
  return (blocks + per - 1) / per;
}

int router_topk_max_groups() { return kRouterMaxGroups; }

bool router_topk_fused_permutes(int tokens) {
  return tokens >= 1 && tokens <= kRouterTokens;  // one token group: its last CTA holds every assignment
}

cudaError_t router_topk_fused_launch(const __nv_bfloat16* x, const float* wr, const float* bias, float* logits_out,
                                     int tokens, int hidden, int experts, int top_k, int32_t* idx, float* w,
                                     float* partial, int* counters, cudaStream_t s, const RouterPermOut* perm) {
  if (tokens == 0) return cudaSuccess;
  if (!router_topk_fused_supported(hidden, experts, top_k)) return cudaErrorInvalidValue;
  const int groups = (tokens + kRouterTokens - 1) / kRouterTokens;
  if (groups > kRouterMaxGroups) return cudaErrorInvalidValue;
  if (perm && !router_topk_fused_permutes(tokens)) return cudaErrorInvalidValue;
  const RouterPermOut po = perm ? *perm : RouterPermOut{};
  const int slices = router_topk_slices(tokens, hidden, experts);
  const int kslice = ((hidden / 128 + slices - 1) / slices) * 128;
  const dim3 grid((experts + kRouterExpertsPerCta - 1) / kRouterExpertsPerCta, slices, groups);
  const int vpt = (experts + 31) / 32;
  cudaError_t e = cudaSuccess;
#define NKI_RTS(V)                                                                                           \
  e = launch_pdl(router_topk_split_kernel<V>, grid, dim3(256), 0, s, x, wr, bias, logits_out, tokens, hidden,      \
                 experts, top_k, idx, w, partial, counters, kslice, po)
  if (vpt <= 1) NKI_RTS(1);
  else if (vpt <= 2) NKI_RTS(2);
  else if (vpt <= 4) NKI_RTS(4);
  else NKI_RTS(8);
#undef NKI_RTS
  return e;
}

bool router_topk_cluster_permutes(int tokens, int top_k) {
  return tokens >= 1 && static_cast<long long>(tokens) * top_k <= kPermuteSmall;
}

cudaError_t router_topk_cluster_launch(const __nv_bfloat16* x, const float* wr, const float* bias, float* logits_out,
                                     int tokens, int hidden, int experts, int top_k, int32_t* idx, float* w,
                                     cudaStream_t s, int* counter, const RouterPermOut* perm) {
  if (tokens == 0) return cudaSuccess;
  if (!router_topk_fused_supported(hidden, experts, top_k)) return cudaErrorInvalidValue;
  if (perm && (!counter || !router_topk_cluster_permutes(tokens, top_k))) return cudaErrorInvalidValue;
  const RouterPermOut po = perm ? *perm : RouterPermOut{};
  const size_t smem = static_cast<size_t>(kRouterCluster) * hidden * sizeof(__nv_bfloat16);
  const unsigned grid = static_cast<unsigned>((tokens + kRouterCluster - 1) / kRouterCluster) * kRouterCluster;
  const int eg = (experts + kRouterCluster - 1) / kRouterCluster;
  // the dynamic shared-memory opt-in (the row staging plus the permutation's
  // static tables pass 48 KB), once per kernel and device so that launches
  // can be captured into CUDA graphs
  static std::mutex mu;
  static std::set<std::pair<int, int>> done;  // (EG, device)
  int dev = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return e0;
#define NKI_RTC(EGV)                                                                                         \
  do {                                                                                                      \
    auto k = router_topk_cluster_kernel<EGV>;                                                               \
    {                                                                                                       \
      std::lock_guard<std::mutex> lock(mu);                                                                 \
      if (!done.count({EGV, dev})) {                                                                        \
        cudaFuncAttributes fa{};                                                                            \
        int optin = 0;                                                                                      \
        cudaError_t e = cudaFuncGetAttributes(&fa, k);                                                      \
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev); \
        if (e == cudaSuccess)                                                                               \
          e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,                          \
                                   optin - static_cast<int>(fa.sharedSizeBytes));                           \
        if (e != cudaSuccess) return e;                                                                     \
        done.insert({EGV, dev});                                                                            \
      }                                                                                                     \
    }                                                                                                       \
    k<<<grid, 256, smem, s>>>(x, wr, bias, logits_out, tokens, hidden, experts, top_k, idx, w, counter, po);  \
  } while (0)
  if (eg <= 4) NKI_RTC(4);
  else if (eg <= 8) NKI_RTC(8);
  else if (eg <= 16) NKI_RTC(16);
  else NKI_RTC(32);
#undef NKI_RTC
  return cudaGetLastError();
}

cudaError_t topk_softmax_launch(const float* logits, int tokens, int experts, int top_k, int32_t* idx, float* w,
                                cudaStream_t s) {
  return topk_softmax_partials_launch(logits, 1, nullptr, nullptr, tokens, experts, top_k, idx, w, s);
}

cudaError_t topk_softmax_partials_launch(const float* partial, int splits, const float* bias, float* logits_out,
                                         int tokens, int experts, int top_k, int32_t* idx, float* w, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (top_k < 1 || top_k > 32 || top_k > experts || experts > 256 || splits < 1 || splits > 8)
    return cudaErrorInvalidValue;
  const int wpb = 8;
  const unsigned blocks = static_cast<unsigned>((tokens + wpb - 1) / wpb);
  const int vpt = (experts + 31) / 32;
#define NKI_TOPK(V)                                                                                          \
  topk_softmax_kernel<V><<<blocks, wpb * 32, 0, s>>>(partial, splits, bias, logits_out, tokens, experts, top_k, \
                                                     idx, w)
  if (vpt <= 1) NKI_TOPK(1);
  else if (vpt <= 2) NKI_TOPK(2);
  else if (vpt <= 4) NKI_TOPK(4);
  else NKI_TOPK(8);
#undef NKI_TOPK
  return cudaGetLastError();
}


size_t router_tc_smem_bytes(int eh) {
  return eh == 128 ? static_cast<size_t>(RtShape<128>::kStages) * RtShape<128>::kStageBytes + 1024
                   : static_cast<size_t>(RtShape<64>::kStages) * RtShape<64>::kStageBytes + 1024;
}

bool router_tc_supported(long long T, int H, int E, bool norm) {
  return E == kRtE && H % kRtBK == 0 && H >= kRtBK && T > 0 && (!norm || H <= 8 * 32 * 8);
}

namespace {
// the dynamic shared-memory opt-in, once per kernel and device (not per
// launch, so launches can be captured into CUDA graphs)
template <bool kNorm, int EH>
cudaError_t router_tc_opt_in(size_t smem) {
  static std::mutex mu;
  static std::set<int> done;  // devices
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (!done.count(dev)) {
    e = cudaFuncSetAttribute(router_tc_kernel<kNorm, EH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    done.insert(dev);
  }
  return cudaSuccess;
}

template <bool kNorm, int EH>
cudaError_t router_tc_run(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const __nv_bfloat16* h,
                          const void* norm_w, int norm_w_dtype, float eps, __nv_bfloat16* x_out, const float* bias,
                          float* logits_out, long long T, int H, int* status, cudaStream_t s) {
  const size_t smem = router_tc_smem_bytes(EH);
  const cudaError_t e = router_tc_opt_in<kNorm, EH>(smem);
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>((kRtE / EH) * ((T + kRtRows - 1) / kRtRows));
  router_tc_kernel<kNorm, EH><<<grid, kRtThreads, smem, s>>>(tmap_x, tmap_w, h, norm_w, norm_w_dtype, eps, x_out,
                                                              bias, logits_out, static_cast<int>(T), H, status);
  return cudaGetLastError();
}
}  // namespace

cudaError_t router_tc_launch(const CUtensorMap& tmap_x, const CUtensorMap& tmap_w, const __nv_bfloat16* h,
                             const void* norm_w, int norm_w_dtype, float eps, __nv_bfloat16* x_out, const float* bias,
                             float* logits_out, long long T, int H, int* status, cudaStream_t s, int experts_per_cta) {
  const bool norm = h != nullptr;
  if (!router_tc_supported(T, H, kRtE, norm) || !logits_out || (norm && (!norm_w || !x_out)) ||
      (experts_per_cta != 64 && experts_per_cta != 128))
    return cudaErrorInvalidValue;
  if (experts_per_cta == 64)
    return norm ? router_tc_run<true, 64>(tmap_x, tmap_w, h, norm_w, norm_w_dtype, eps, x_out, bias, logits_out, T,
                                          H, status, s)
                : router_tc_run<false, 64>(tmap_x, tmap_w, nullptr, nullptr, 0, 0.f, nullptr, bias, logits_out, T,
                                           H, status, s);
  return norm ? router_tc_run<true, 128>(tmap_x, tmap_w, h, norm_w, norm_w_dtype, eps, x_out, bias, logits_out, T, H,
                                         status, s)
              : router_tc_run<false, 128>(tmap_x, tmap_w, nullptr, nullptr, 0, 0.f, nullptr, bias, logits_out, T, H,
                                          status, s);
}
}  // namespace nkimoe
