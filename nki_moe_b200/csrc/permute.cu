// K3: permutation of the T*K (token, slot) assignments by expert, and the
// row movers around the expert GEMMs.
//
// Order contract (nki_moe_integrated.py:450-467): slot k outer, expert inner,
// tokens ascending, i.e. inside expert e the rows are sorted by (k, t).  The
// assignments are walked in k-major order j = k*T + t; the permutation is a
// stable counting sort of j by expert:
//   1. count:   per 256-assignment chunk, per-expert counts        [C][E]
//   2. scan:    per expert, exclusive prefix over chunks + totals   [C][E], [E]
//   3. scatter: per chunk, expert offset + chunk base + rank of the
//               assignment among earlier same-expert assignments of its chunk
//               (warp match_any + popc, then per-warp counts).
// No host synchronisation: the GEMMs read expert_offsets on the device.
#include "kernels.h"
#include "permute_small.cuh"

namespace nkimoe {

namespace {

template <typename IdxT>
__global__ void __launch_bounds__(kPermuteChunk) permute_count_kernel(const IdxT* __restrict__ idx, int T, int K,
                                                                      int E, int* __restrict__ chunk_counts,
                                                                      int* status) {
  __shared__ int cnt[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const long long j = static_cast<long long>(blockIdx.x) * kPermuteChunk + threadIdx.x;
  if (j < static_cast<long long>(T) * K) {
    const int e = load_expert(idx, j, T, K, E, status);
    if (e >= 0) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_counts[static_cast<long long>(blockIdx.x) * E + e] = cnt[e];
}

// One block per expert: exclusive scan of that expert's chunk counts.
__global__ void __launch_bounds__(256) permute_scan_kernel(const int* __restrict__ chunk_counts, int C, int E,
                                                           int* __restrict__ chunk_base, int* __restrict__ totals) {
  __shared__ int warp_tot[8];
  const int e = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int running = 0;
  for (int c0 = 0; c0 < C; c0 += 256) {
    const int c = c0 + threadIdx.x;
    const int v = c < C ? chunk_counts[static_cast<long long>(c) * E + e] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      before += w < warp ? warp_tot[w] : 0;
      all += warp_tot[w];
    }
    if (c < C) chunk_base[static_cast<long long>(c) * E + e] = running + before + incl - v;
    running += all;
    __syncthreads();
  }
  if (threadIdx.x == 0) totals[e] = running;
}

template <typename IdxT>
__global__ void __launch_bounds__(kPermuteChunk) permute_scatter_kernel(
    const IdxT* __restrict__ idx, int T, int K, int E, const int* __restrict__ chunk_base,
    const int* __restrict__ totals, int32_t* __restrict__ row_token, int32_t* __restrict__ row_slot,
    int32_t* __restrict__ slot_row, int32_t* __restrict__ expert_offsets, const float* __restrict__ slot_weight,
    float* __restrict__ row_weight, int* status) {
  constexpr int kWarps = kPermuteChunk / 32;
  __shared__ int offs[kMaxExperts + 1];
  __shared__ int wcnt[kWarps][kMaxExperts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (warp == 0) {  // expert offsets = exclusive scan of totals
    int run = 0;
    for (int b = 0; b < E; b += 32) {
      const int e = b + lane;
      const int v = e < E ? totals[e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (e < E) offs[e] = run + incl - v;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) offs[E] = run;
  }
  for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) wcnt[i / E][i % E] = 0;
  __syncthreads();
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e <= E; e += blockDim.x) expert_offsets[e] = offs[e];

  const long long j = static_cast<long long>(blockIdx.x) * kPermuteChunk + threadIdx.x;
  const bool valid = j < static_cast<long long>(T) * K;
  int e = -1;
  if (valid) {
    // range errors were flagged by the count pass
    const long long k = j / T, t = j % T;
    const long long ev = static_cast<long long>(idx[t * K + k]);
    e = (ev >= 0 && ev < E) ? static_cast<int>(ev) : -1;
  }
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
  __syncthreads();
  if (!valid) return;
  const long long k = j / T, t = j % T;
  const long long slot = t * K + k;
  if (e < 0) {
    slot_row[slot] = -1;
    return;
  }
  int before = 0;
  for (int w = 0; w < warp; ++w) before += wcnt[w][e];
  const int pos = offs[e] + chunk_base[static_cast<long long>(blockIdx.x) * E + e] + before + rank;
  row_token[pos] = static_cast<int32_t>(t);
  row_slot[pos] = static_cast<int32_t>(slot);
  slot_row[slot] = pos;
  if (row_weight) row_weight[pos] = slot_weight[slot];
  (void)status;
}

// The permutation for few assignments (T*K <= kPermuteSmall, decode) in one
// CTA (permute_small.cuh): a block call pays one launch instead of three.
template <typename IdxT>
__global__ void __launch_bounds__(kPermuteChunk) permute_small_kernel(
    const IdxT* __restrict__ idx, int T, int K, int E, int32_t* __restrict__ row_token,
    int32_t* __restrict__ row_slot, int32_t* __restrict__ slot_row, int32_t* __restrict__ expert_offsets,
    const float* __restrict__ slot_weight, float* __restrict__ row_weight, int* status) {
  pdl_launch_dependents();
  pdl_wait();
  permute_small_cta<IdxT>(idx, T, K, E, row_token, row_slot, slot_row, expert_offsets, slot_weight, row_weight,
                          status);
}

// x_perm[r] = x[row_token[r]] for r < expert_offsets[E].  One warp per row;
// each lane keeps up to 8 independent 16-byte loads in flight (a 4 KB row of
// H = 2048 is one pass).
__global__ void __launch_bounds__(256) gather_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const int32_t* __restrict__ row_token,
                                                          const int32_t* __restrict__ expert_offsets, int E,
                                                          __nv_bfloat16* __restrict__ xp, long long max_rows,
                                                          int H) {
  const int chunks = H >> 3;  // 16-byte chunks per row
  const int lane = threadIdx.x & 31;
  pdl_launch_dependents();
  pdl_wait();
  const long long rows = min(static_cast<long long>(expert_offsets[E]), max_rows);
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += nwarps) {
    const long long t = row_token[r];
    const uint4* src = reinterpret_cast<const uint4*>(x + t * H);
    uint4* dst = reinterpret_cast<uint4*>(xp + r * H);
    for (int c0 = lane; c0 < chunks; c0 += 256) {
      uint4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + 32 * j < chunks) v[j] = src[c0 + 32 * j];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (c0 + 32 * j < chunks) __stcs(dst + c0 + 32 * j, v[j]);  // streaming: keeps x resident in L2
    }
  }
}

// out[t] = sum_k w[t,k] * y[slot_row[t*K+k]] in fp32 with k ascending (the
// accumulation order of nki_moe_integrated.py:482-494).  When slot_weight is
// null the rows already carry their routing weight.  One thread per 16-byte
// column chunk of a token (32-bit index math; T * H / 8 < 2^31), its K row
// loads in flight together; y rows are read once, so they are loaded with
// the evict-first hint.
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ y,
                                                      const int32_t* __restrict__ slot_row,
                                                      const float* __restrict__ slot_weight,
                                                      __nv_bfloat16* __restrict__ out, int T, int K, int H) {
  const uint32_t chunks = static_cast<uint32_t>(H) >> 3;
  const uint32_t n = static_cast<uint32_t>(T) * chunks;
  pdl_launch_dependents();
  pdl_wait();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t t = i / chunks;
    const uint32_t c = i - t * chunks;
    float acc[8] = {};
    for (int k0 = 0; k0 < K; k0 += 8) {
      uint4 u[8];
      int rr[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        rr[j] = k0 + j < K ? slot_row[t * K + k0 + j] : -1;
        if (rr[j] >= 0) u[j] = __ldcs(reinterpret_cast<const uint4*>(y + static_cast<long long>(rr[j]) * H) + c);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (rr[j] < 0) continue;
        const float wk = slot_weight ? slot_weight[t * K + k0 + j] : 1.f;
        const float2 a = unpack_bf16x2(u[j].x), b = unpack_bf16x2(u[j].y), cc = unpack_bf16x2(u[j].z),
                     d = unpack_bf16x2(u[j].w);
        acc[0] = fmaf(wk, a.x, acc[0]);
        acc[1] = fmaf(wk, a.y, acc[1]);
        acc[2] = fmaf(wk, b.x, acc[2]);
        acc[3] = fmaf(wk, b.y, acc[3]);
        acc[4] = fmaf(wk, cc.x, acc[4]);
        acc[5] = fmaf(wk, cc.y, acc[5]);
        acc[6] = fmaf(wk, d.x, acc[6]);
        acc[7] = fmaf(wk, d.y, acc[7]);
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + static_cast<long long>(t) * H)[c] = o;
  }
}

// Sum over the leading top-k axis of [K, T, H] (nki_moe_integrated.py:209-251).
__global__ void __launch_bounds__(256) aggregate_kernel(const __nv_bfloat16* __restrict__ eo,
                                                        __nv_bfloat16* __restrict__ out, int K, long long T, int H) {
  const int chunks = H >> 3;
  const long long n = T * chunks;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float acc[8] = {};
    for (int k = 0; k < K; ++k) {
      const uint4 u = reinterpret_cast<const uint4*>(eo + static_cast<long long>(k) * T * H)[i];
      const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), cc = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
      acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
      acc[4] += cc.x; acc[5] += cc.y; acc[6] += d.x; acc[7] += d.y;
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

// silu(gate) * up over a [M, 2N] gate|up split (nki_moe_integrated.py:87-139).
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* __restrict__ gu,
                                                     __nv_bfloat16* __restrict__ out, long long M, int N) {
  const long long n = M * N;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / N;
    const int c = static_cast<int>(i % N);
    const float g = __bfloat162float(gu[r * 2 * N + c]);
    const float u = __bfloat162float(gu[r * 2 * N + N + c]);
    out[i] = __float2bfloat16_rn(silu_f(g) * u);
  }
}

__global__ void offsets_to_counts_kernel(const int32_t* __restrict__ offsets, int32_t* __restrict__ counts, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) counts[i] = offsets[i + 1] - offsets[i];
}

// One block of 512 threads: exclusive scan of n <= 512 counts.
__global__ void __launch_bounds__(512) counts_to_offsets_kernel(const int32_t* __restrict__ counts,
                                                                int32_t* __restrict__ offsets, int n) {
  __shared__ int warp_tot[16];
  const int i = threadIdx.x, lane = i & 31, warp = i >> 5;
  const int v = i < n ? counts[i] : 0;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int x = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += x;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int before = 0;
  for (int w = 0; w < warp; ++w) before += warp_tot[w];
  if (i < n) offsets[i + 1] = before + incl;
  if (i == 0) offsets[0] = 0;
}

// Expert-parallel dispatch, step 1: dest[t][d] = d if one of token t's
// experts lives on rank d (experts [d*El, (d+1)*El)), else -1.  The
// permutation kernels then group the (token, rank) pairs by rank, tokens
// ascending.
__global__ void ep_dest_kernel(const int32_t* __restrict__ idx, int T, int K, int P, int El,
                               int32_t* __restrict__ dest) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(T) * P) return;
  const long long t = i / P;
  const int d = static_cast<int>(i % P);
  int hit = 0;
  for (int k = 0; k < K; ++k) {
    const int e = idx[t * K + k];
    hit |= (e >= d * El && e < (d + 1) * El);
  }
  dest[i] = hit ? d : -1;
}

// Step 2: for send row r = (token t, rank d) the K slots as rank d sees them:
// local expert id (or -1 when slot k's expert lives elsewhere) and weight.
__global__ void ep_slots_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w,
                                const int32_t* __restrict__ row_token, const int32_t* __restrict__ row_slot,
                                const int32_t* __restrict__ rank_offsets, int P, int K, int El,
                                int32_t* __restrict__ slots, float* __restrict__ wts) {
  const long long rows = rank_offsets[P];
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows * K;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / K;
    const int k = static_cast<int>(i % K);
    const long long t = row_token[r];
    const int d = row_slot[r] % P;
    const int e = idx[t * K + k];
    const bool local = e >= d * El && e < (d + 1) * El;
    slots[i] = local ? e - d * El : -1;
    wts[i] = local ? w[t * K + k] : 0.f;
  }
}

unsigned grid_for(long long work, int threads) {
  const long long b = (work + threads - 1) / threads;
  const long long cap = static_cast<long long>(device_sm_count()) * 16;
  return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

size_t permute_scratch_bytes(long long tokens, int top_k, int experts) {
  const long long C = (tokens * top_k + kPermuteChunk - 1) / kPermuteChunk;
  // chunk_counts [C][E] + chunk_base [C][E] + totals [E]
  return static_cast<size_t>((2 * C * experts + experts) * sizeof(int));
}

cudaError_t permute_launch(const void* idx, int idx_dtype, int tokens, int top_k, int experts, int32_t* row_token,
                           int32_t* row_slot, int32_t* slot_row, int32_t* expert_offsets, void* scratch,
                           int* status, cudaStream_t s, const float* slot_weight, float* row_weight) {
  if (experts > kMaxExperts || experts < 1) return cudaErrorInvalidValue;
  const long long TK = static_cast<long long>(tokens) * top_k;
  const int C = static_cast<int>((TK + kPermuteChunk - 1) / kPermuteChunk);
  int* chunk_counts = static_cast<int*>(scratch);
  int* chunk_base = chunk_counts + static_cast<long long>(C) * experts;
  int* totals = chunk_base + static_cast<long long>(C) * experts;
  if (C == 0) {
    cudaMemsetAsync(expert_offsets, 0, sizeof(int32_t) * (experts + 1), s);
    return cudaGetLastError();
  }
  if (TK <= kPermuteSmall) {
    if (idx_dtype == kI64)
      return launch_pdl(permute_small_kernel<long long>, dim3(1), dim3(kPermuteChunk), 0, s,
                        static_cast<const long long*>(idx), tokens, top_k, experts, row_token, row_slot, slot_row,
                        expert_offsets, slot_weight, row_weight, status);
    return launch_pdl(permute_small_kernel<int32_t>, dim3(1), dim3(kPermuteChunk), 0, s,
                      static_cast<const int32_t*>(idx), tokens, top_k, experts, row_token, row_slot, slot_row,
                      expert_offsets, slot_weight, row_weight, status);
  }
  if (idx_dtype == kI64) {
    permute_count_kernel<long long><<<C, kPermuteChunk, 0, s>>>(static_cast<const long long*>(idx), tokens, top_k,
                                                                experts, chunk_counts, status);
  } else {
    permute_count_kernel<int32_t><<<C, kPermuteChunk, 0, s>>>(static_cast<const int32_t*>(idx), tokens, top_k,
                                                              experts, chunk_counts, status);
  }
  permute_scan_kernel<<<experts, 256, 0, s>>>(chunk_counts, C, experts, chunk_base, totals);
  if (idx_dtype == kI64) {
    permute_scatter_kernel<long long><<<C, kPermuteChunk, 0, s>>>(static_cast<const long long*>(idx), tokens, top_k,
                                                                  experts, chunk_base, totals, row_token, row_slot,
                                                                  slot_row, expert_offsets, slot_weight, row_weight,
                                                                  status);
  } else {
    permute_scatter_kernel<int32_t><<<C, kPermuteChunk, 0, s>>>(static_cast<const int32_t*>(idx), tokens, top_k,
                                                                experts, chunk_base, totals, row_token, row_slot,
                                                                slot_row, expert_offsets, slot_weight, row_weight,
                                                                status);
  }
  return cudaGetLastError();
}

cudaError_t gather_rows_launch(const __nv_bfloat16* x, const int32_t* row_token, const int32_t* expert_offsets,
                               int experts, __nv_bfloat16* x_perm, long long max_rows, int hidden, cudaStream_t s) {
  if (max_rows == 0) return cudaSuccess;
  return launch_pdl(gather_rows_kernel, dim3(grid_for(max_rows * 32, 256)), dim3(256), 0, s, x, row_token,
                    expert_offsets, experts, x_perm, max_rows, hidden);
}

cudaError_t combine_launch(const __nv_bfloat16* y, const int32_t* slot_row, const float* slot_weight,
                           __nv_bfloat16* out, int tokens, int top_k, int hidden, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (static_cast<long long>(tokens) * (hidden / 8) >= (1LL << 31)) return cudaErrorInvalidValue;
  return launch_pdl(combine_kernel, dim3(grid_for(static_cast<long long>(tokens) * (hidden / 8), 256)), dim3(256), 0,
                    s, y, slot_row, slot_weight, out, tokens, top_k, hidden);
}

cudaError_t offsets_to_counts_launch(const int32_t* offsets, int32_t* counts, int n, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  offsets_to_counts_kernel<<<(n + 255) / 256, 256, 0, s>>>(offsets, counts, n);
  return cudaGetLastError();
}

cudaError_t counts_to_offsets_launch(const int32_t* counts, int32_t* offsets, int n, cudaStream_t s) {
  if (n <= 0 || n > 512) return cudaErrorInvalidValue;
  counts_to_offsets_kernel<<<1, 512, 0, s>>>(counts, offsets, n);
  return cudaGetLastError();
}

cudaError_t ep_dest_launch(const int32_t* idx, int T, int K, int P, int El, int32_t* dest, cudaStream_t s) {
  const long long n = static_cast<long long>(T) * P;
  if (n == 0) return cudaSuccess;
  ep_dest_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(idx, T, K, P, El, dest);
  return cudaGetLastError();
}

cudaError_t ep_slots_launch(const int32_t* idx, const float* w, const int32_t* row_token, const int32_t* row_slot,
                            const int32_t* rank_offsets, long long max_rows, int P, int K, int El, int32_t* slots,
                            float* wts, cudaStream_t s) {
  if (max_rows == 0) return cudaSuccess;
  ep_slots_kernel<<<grid_for(max_rows * K, 256), 256, 0, s>>>(idx, w, row_token, row_slot, rank_offsets, P, K, El,
                                                              slots, wts);
  return cudaGetLastError();
}

cudaError_t aggregate_launch(const __nv_bfloat16* eo, __nv_bfloat16* out, int top_k, long long tokens, int hidden,
                             cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  aggregate_kernel<<<grid_for(tokens * (hidden / 8), 256), 256, 0, s>>>(eo, out, top_k, tokens, hidden);
  return cudaGetLastError();
}

cudaError_t swiglu_launch(const __nv_bfloat16* gate_up, __nv_bfloat16* out, long long rows, int n, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  swiglu_kernel<<<grid_for(rows * n, 256), 256, 0, s>>>(gate_up, out, rows, n);
  return cudaGetLastError();
}

}  // namespace nkimoe
