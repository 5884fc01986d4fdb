// Decode-step attention over a KV cache (grouped-query attention, head_dim
// 128), fused with what feeds it: the q/k RMSNorm + rotate-half RoPE of the
// step's token and the store of its key and value into the cache.
//
// Reference: nki_attention.py:252-373 (nki_flash_attention_decode: one query
// token against the cached keys/values, online softmax :333-359) and the
// attention block of qwen_with_nki.py:330-350 (q/k NKIRMSNorm per head, then
// RoPE; HF Qwen3-MoE order and rotate-half convention).
//
// Split-KV ("flash decoding"): CTA (c, j, b) takes kv head j of sequence b
// and the cache positions [c*chunk, min((c+1)*chunk, pos+1)).  It computes
// the grp = nq/nkv query heads of kv head j itself (norm + RoPE + scale), so
// no CTA waits for another; the CTA whose chunk holds `pos` also normalises,
// rotates and stores the new key and stores the new value.  Each CTA leaves
// (m, l, o) per head in the workspace; the last CTA of (b, j) to finish
// (device-scope counter, no spinning) merges them and writes the bf16 output.
// The counter is left at zero for the next call.
#include "kernels.h"
#include "rope.cuh"

namespace nkimoe {

namespace {

constexpr int kAttnWarps = 8;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kSub = 64;          // cache positions per block (one MMA n-tile of 8 per warp)
constexpr int kMaxSplits = 32;    // CTAs per (sequence, kv head)
constexpr int kMaxGroup = 16;     // query heads per kv head: the MMA's 16 rows
constexpr int kPartStride = 132;  // floats per (split, head) partial: o[128], m, l, pad
static_assert(kMaxSplits <= 32, "the merge keeps one split per lane");
constexpr int kRowK = kHeadDim + 8;  // padded smem row (272 B): conflict-free ldmatrix
constexpr int kRowP = kSub + 8;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnParams {
  const __nv_bfloat16* qkv;  // [B, (nq + 2 nkv) * 128]
  const void* qw;
  const void* kw;
  const long long* positions;
  __nv_bfloat16* k_cache;  // [B, nkv, max_seq, 128]
  __nv_bfloat16* v_cache;
  __nv_bfloat16* out;  // [B, nq * 128]
  float* part;         // [B, nkv, nsplit, grp, kPartStride]
  int* counters;       // [B, nkv]
  int* status;
  long long pos_stride;
  int w_dtype, nq, nkv, grp, max_seq, chunk, nsplit;
  float theta, eps, scale_log2;
};

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_trans(const void* p, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// D[16x8] += A[16x16] (row) * B[16x8] (col), bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One CTA: kv head j of sequence b, cache positions [c*chunk, ...).  The two
// small products of a 64-position block run as warp MMAs (m16n8k16, bf16 in,
// fp32 accumulate): S[16 heads x 64 positions] = Q K^T with warp w taking
// positions 8w..8w+7, then O[16 heads x 128] += P V with warp w taking head
// dims 16w..16w+15.  Rows of Q beyond the group's heads are zero.
__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(AttnParams p) {
  constexpr int D = kHeadDim;
  const int c = blockIdx.x, j = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;  // MMA fragment row group / column pair
  pdl_launch_dependents();
  pdl_wait();
  // the step's query rows (and the key / value row for warps 0 / 1) do not
  // depend on the position: their loads go out first
  const long long row_len = static_cast<long long>(p.nq + 2 * p.nkv) * D;
  const __nv_bfloat16* qrow = p.qkv + b * row_len;
  float qv[2][4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = warp + h * kAttnWarps;
    if (i < p.grp) head_load4(qrow + static_cast<long long>(j * p.grp + i) * D + lane * 4, qv[h]);
  }
  float kvv[4] = {0.f, 0.f, 0.f, 0.f};
  if (warp < 2) head_load4(qrow + static_cast<long long>(p.nq + warp * p.nkv + j) * D + lane * 4, kvv);
  const long long pos = p.positions[b * p.pos_stride];
  if (pos < 0 || pos >= p.max_seq) {  // nothing is read or written for this sequence
    if (c == 0 && threadIdx.x == 0) atomicOr(p.status, kDevErrBadIndex);
    return;
  }
  const int ipos = static_cast<int>(pos);
  const int n_act = ipos / p.chunk + 1;  // CTAs of (b, j) with work
  if (c >= n_act) return;
  const int lo = c * p.chunk;
  const int hi = min(lo + p.chunk, ipos + 1);

  __shared__ __align__(16) __nv_bfloat16 ks[kSub][kRowK];
  __shared__ __align__(16) __nv_bfloat16 vs[kSub][kRowK];
  __shared__ __align__(16) __nv_bfloat16 qs[kMaxGroup][kRowK];
  __shared__ __align__(16) __nv_bfloat16 ps[kMaxGroup][kRowP];
  __shared__ float red_m[kAttnWarps][kMaxGroup];
  __shared__ float red_l[kAttnWarps][kMaxGroup];
  __shared__ float2 rope_tab[D / 2];
  __shared__ int s_last;

  const long long cache_base = (static_cast<long long>(b) * p.nkv + j) * p.max_seq * D;
  const __nv_bfloat16* kc = p.k_cache + cache_base;
  const __nv_bfloat16* vc = p.v_cache + cache_base;

  // stage rows [s0, s0 + n) of K and V (16-byte pieces, 16 per row); rows
  // n..63 are zero-filled and the row at `pos` comes from registers
  auto stage = [&](int s0, int n) {
    for (int q = threadIdx.x; q < 2 * kSub * 16; q += kAttnThreads) {
      const int which = q >> 10;  // 0: K, 1: V (kSub * 16 = 1024 pieces each)
      const int r = (q >> 4) & (kSub - 1);
      const int piece = q & 15;
      if (s0 + r == ipos) continue;
      const bool live = r < n;
      const __nv_bfloat16* src = (which ? vc : kc) + static_cast<long long>(live ? s0 + r : lo) * D + piece * 8;
      __nv_bfloat16* dst = (which ? &vs[r][0] : &ks[r][0]) + piece * 8;
      cp_async_16(smem_u32(dst), src, live ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  stage(lo, min(kSub, hi - lo));  // in flight while the queries are prepared

  // RoPE cos / sin of this position, one frequency per thread
  if (threadIdx.x < D / 2) {
    float cs, sn;
    rope_cs(static_cast<float>(pos), threadIdx.x, p.theta, cs, sn);
    rope_tab[threadIdx.x] = make_float2(cs, sn);
  }
  __syncthreads();
  float tc[4], tsn[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 v = rope_tab[(lane * 4 + e) & (D / 2 - 1)];
    tc[e] = v.x;
    tsn[e] = v.y;
  }
  // queries j*grp + i: normalised, rotated, scaled by softmax_scale * log2(e)
  // (the softmax runs in base 2) and rounded to bf16 for the MMA
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = warp + h * kAttnWarps;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    if (i < p.grp) {
      float nv[4];
      head_rmsnorm(qv[h], p.qw, p.w_dtype, p.eps, lane, nv);
      head_rope(nv, tc, tsn, lane, o);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] *= p.scale_log2;
    }
    head_store4(&qs[i][lane * 4], o);
  }
  // the new token's key (normalised, rotated, rounded to bf16) and value
  const bool owns_pos = (c == n_act - 1);
  uint2 newrow = make_uint2(0u, 0u);
  if (owns_pos && warp < 2) {
    if (warp == 0) {
      float nv[4], o[4];
      head_rmsnorm(kvv, p.kw, p.w_dtype, p.eps, lane, nv);
      head_rope(nv, tc, tsn, lane, o);
      newrow.x = pack_bf16x2(o[0], o[1]);
      newrow.y = pack_bf16x2(o[2], o[3]);
      *reinterpret_cast<uint2*>(p.k_cache + cache_base + pos * D + lane * 4) = newrow;
    } else {  // the value row, bit for bit (bf16 -> fp32 -> bf16 is exact)
      newrow.x = pack_bf16x2(kvv[0], kvv[1]);
      newrow.y = pack_bf16x2(kvv[2], kvv[3]);
      *reinterpret_cast<uint2*>(p.v_cache + cache_base + pos * D + lane * 4) = newrow;
    }
  }

  // running softmax state of heads g and g + 8 (identical in every thread
  // that holds them), output accumulators for head dims 16w + 8nt + 2t, +1
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};

  for (int s0 = lo; s0 < hi; s0 += kSub) {
    const int n = min(kSub, hi - s0);
    if (s0 != lo) stage(s0, n);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (owns_pos && warp < 2 && ipos >= s0 && ipos < s0 + n)
      *reinterpret_cast<uint2*>((warp == 0 ? &ks[ipos - s0][0] : &vs[ipos - s0][0]) + lane * 4) = newrow;
    __syncthreads();

    // S = Q K^T for positions 8w .. 8w+7
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int kk = 0; kk < D / 16; kk += 2) {
      uint32_t a0[4], a1[4], bk[4];
      ldsm_x4(&qs[(lane & 7) + ((lane >> 3) & 1) * 8][kk * 16 + (lane >> 4) * 8], a0);
      ldsm_x4(&qs[(lane & 7) + ((lane >> 3) & 1) * 8][(kk + 1) * 16 + (lane >> 4) * 8], a1);
      ldsm_x4(&ks[warp * 8 + (lane & 7)][kk * 16 + (lane >> 3) * 8], bk);
      mma_16816(sc, a0, bk[0], bk[1]);
      mma_16816(sc, a1, bk[2], bk[3]);
    }
    // sc[0..1]: head g, positions 8w + 2t, +1; sc[2..3]: head g + 8
    const int p0 = warp * 8 + 2 * t;
    if (p0 >= n) sc[0] = sc[2] = -INFINITY;
    if (p0 + 1 >= n) sc[1] = sc[3] = -INFINITY;
    float wm[2] = {fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3])};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      wm[h] = fmaxf(wm[h], __shfl_xor_sync(0xffffffffu, wm[h], 1));
      wm[h] = fmaxf(wm[h], __shfl_xor_sync(0xffffffffu, wm[h], 2));
    }
    if (t == 0) {
      red_m[warp][g] = wm[0];
      red_m[warp][g + 8] = wm[1];
    }
    __syncthreads();
    float mnew[2], alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = m_run[h];
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, red_m[w][g + 8 * h]);
      mnew[h] = mx;
      alpha[h] = exp2f(m_run[h] - mx);  // 0 on the first block (m_run = -inf)
    }
    // P = exp2(S - m) in bf16 (its rounded values are also what l sums)
    float ls[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_bfloat162 pp = __floats2bfloat162_rn(exp2f(sc[2 * h] - mnew[h]), exp2f(sc[2 * h + 1] - mnew[h]));
      *reinterpret_cast<__nv_bfloat162*>(&ps[g + 8 * h][p0]) = pp;
      const float2 pf = __bfloat1622float2(pp);
      ls[h] = pf.x + pf.y;
      ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], 1);
      ls[h] += __shfl_xor_sync(0xffffffffu, ls[h], 2);
    }
    if (t == 0) {
      red_l[warp][g] = ls[0];
      red_l[warp][g + 8] = ls[1];
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float lsum = 0.f;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) lsum += red_l[w][g + 8 * h];
      l_run[h] = l_run[h] * alpha[h] + lsum;
      m_run[h] = mnew[h];
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      acc[nt][0] *= alpha[0];
      acc[nt][1] *= alpha[0];
      acc[nt][2] *= alpha[1];
      acc[nt][3] *= alpha[1];
    }
    // O += P V for head dims 16w .. 16w+15
#pragma unroll
    for (int kk = 0; kk < kSub / 16; ++kk) {
      uint32_t a[4], bv[4];
      ldsm_x4(&ps[(lane & 7) + ((lane >> 3) & 1) * 8][kk * 16 + (lane >> 4) * 8], a);
      ldsm_x4_trans(&vs[kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)][warp * 16 + (lane >> 4) * 8], bv);
      mma_16816(acc[0], a, bv[0], bv[1]);
      mma_16816(acc[1], a, bv[2], bv[3]);
    }
    __syncthreads();  // the next block overwrites ks / vs / ps / red_*
  }

  // this thread's outputs: heads g (acc[nt][0..1]) and g + 8 (acc[nt][2..3]),
  // dims warp*16 + nt*8 + 2t, +1
  const long long ob = static_cast<long long>(b) * p.nq * D;
  if (n_act == 1) {  // one CTA: its result is final
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = g + 8 * h;
      if (i >= p.grp) continue;
      const float inv = 1.f / l_run[h];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        *reinterpret_cast<uint32_t*>(p.out + ob + static_cast<long long>(j * p.grp + i) * D + warp * 16 + nt * 8 +
                                     2 * t) = pack_bf16x2(acc[nt][2 * h] * inv, acc[nt][2 * h + 1] * inv);
    }
    return;
  }

  float* part_bj = p.part + (static_cast<long long>(b) * p.nkv + j) * p.nsplit * p.grp * kPartStride;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int i = g + 8 * h;
    if (i >= p.grp) continue;
    float* dst = part_bj + (static_cast<long long>(c) * p.grp + i) * kPartStride;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
      __stcg(reinterpret_cast<float2*>(dst + warp * 16 + nt * 8 + 2 * t), make_float2(acc[nt][2 * h], acc[nt][2 * h + 1]));
    if (warp == 0 && t == 0) __stcg(reinterpret_cast<float2*>(dst + D), make_float2(m_run[h], l_run[h]));
  }
  // publish: the CTA barrier orders every thread's partial stores before
  // thread 0's fence and counter increment (one fence per CTA)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(p.counters + b * p.nkv + j, 1);
    s_last = (done == n_act - 1);
    if (s_last) __threadfence();
  }
  __syncthreads();
  if (!s_last) return;

  // merge the n_act partials of every head in split order: lane s holds split
  // s's (m, l) and its base-2 weight; the partial rows are loaded 4 at a time
  for (int i = warp; i < p.grp; i += kAttnWarps) {
    const float* base = part_bj + static_cast<long long>(i) * kPartStride;
    const long long sstride = static_cast<long long>(p.grp) * kPartStride;
    float2 ml = make_float2(-INFINITY, 0.f);
    if (lane < n_act) ml = __ldcg(reinterpret_cast<const float2*>(base + lane * sstride + D));
    const float mx = warp_max(ml.x);
    const float f = lane < n_act ? exp2f(ml.x - mx) : 0.f;
    const float L = warp_sum(f * ml.y);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < n_act; s0 += 4) {
      float4 ov[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        ov[u] = s0 + u < n_act ? __ldcg(reinterpret_cast<const float4*>(base + (s0 + u) * sstride + lane * 4))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float fu = __shfl_sync(0xffffffffu, f, (s0 + u) & 31);
        o[0] = fmaf(fu, ov[u].x, o[0]);
        o[1] = fmaf(fu, ov[u].y, o[1]);
        o[2] = fmaf(fu, ov[u].z, o[2]);
        o[3] = fmaf(fu, ov[u].w, o[3]);
      }
    }
    const float inv = 1.f / L;
    head_store4(p.out + ob + static_cast<long long>(j * p.grp + i) * D + lane * 4,
                {o[0] * inv, o[1] * inv, o[2] * inv, o[3] * inv});
  }
  if (threadIdx.x == 0) p.counters[b * p.nkv + j] = 0;  // ready for the next call
}

}  // namespace

int decode_attention_chunk(int max_seq) {
  const int subs = (max_seq + kSub - 1) / kSub;
  const int per = (subs + kMaxSplits - 1) / kMaxSplits;
  return per * kSub;
}

size_t decode_attention_workspace_bytes(long long B, int n_heads, int n_kv, int max_seq) {
  const int chunk = decode_attention_chunk(max_seq);
  const long long nsplit = (max_seq + chunk - 1) / chunk;
  const long long grp = n_kv > 0 ? n_heads / n_kv : 0;
  const size_t counters = (sizeof(int) * B * n_kv + 255) & ~static_cast<size_t>(255);
  return 256 + counters + sizeof(float) * B * n_kv * nsplit * grp * kPartStride;
}

cudaError_t decode_attention_launch(const __nv_bfloat16* qkv, const void* qw, const void* kw, int w_dtype,
                                    const long long* positions, long long pos_stride, __nv_bfloat16* k_cache,
                                    __nv_bfloat16* v_cache, __nv_bfloat16* out, int B, int n_heads, int n_kv,
                                    int max_seq, float theta, float eps, float scale, void* workspace,
                                    cudaStream_t s) {
  AttnParams p{};
  p.qkv = qkv;
  p.qw = qw;
  p.kw = kw;
  p.w_dtype = w_dtype;
  p.positions = positions;
  p.pos_stride = pos_stride;
  p.k_cache = k_cache;
  p.v_cache = v_cache;
  p.out = out;
  p.nq = n_heads;
  p.nkv = n_kv;
  p.grp = n_heads / n_kv;
  p.max_seq = max_seq;
  p.chunk = decode_attention_chunk(max_seq);
  p.nsplit = (max_seq + p.chunk - 1) / p.chunk;
  p.theta = theta;
  p.eps = eps;
  p.scale_log2 = scale * kLog2e;
  char* ws = static_cast<char*>(workspace);
  p.status = reinterpret_cast<int*>(ws);
  p.counters = reinterpret_cast<int*>(ws + 256);
  const size_t counters = (sizeof(int) * static_cast<size_t>(B) * n_kv + 255) & ~static_cast<size_t>(255);
  p.part = reinterpret_cast<float*>(ws + 256 + counters);
  if (p.grp > kMaxGroup) return cudaErrorInvalidValue;
  const dim3 grid(p.nsplit, n_kv, B);
  return launch_pdl(decode_attention_kernel, grid, dim3(kAttnThreads), 0, s, p);
}

}  // namespace nkimoe
