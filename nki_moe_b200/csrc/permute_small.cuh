// Stable grouping of a decode batch's (token, slot) assignments by expert in
// one CTA, shared by the permutation kernel and the decode router (which runs
// it in its last CTA when the batch is one token group).  Order: experts
// ascending, (k, t) lexicographic inside an expert (nki_moe_integrated.py:450-467).
#pragma once

#include "kernels.h"

namespace nkimoe {

// A negative id marks an empty slot (skipped); an id >= E is an error.
template <typename IdxT>
__device__ __forceinline__ int load_expert(const IdxT* idx, long long j, int T, int K, int E, int* status) {
  const long long k = j / T, t = j % T;
  const long long e = static_cast<long long>(idx[t * K + k]);
  if (e < 0) return -1;
  if (e >= E) {
    atomicOr(status, kDevErrBadIndex);
    return -1;
  }
  return static_cast<int>(e);
}

// The permutation for few assignments (T*K <= kPermuteSmall, decode) by one
// CTA of kPermuteChunk threads (all of them must call it): every thread
// loads its assignments' expert ids once (assignment j = c * 256 + thread of
// chunk c; k-major: j = k * T + t), the CTA counts and scans them in shared memory,
// then walks the chunks in order with the same warp match_any ranking, adding
// a running per-expert count between chunks.  Bit-identical to the
// count/scan/scatter kernels.
constexpr int kPermuteSmall = 8 * kPermuteChunk;

template <typename IdxT>
__device__ __forceinline__ void permute_small_cta(const IdxT* idx, int T, int K, int E, int32_t* row_token,
                                                  int32_t* row_slot, int32_t* slot_row, int32_t* expert_offsets,
                                                  const float* slot_weight, float* row_weight, int* status) {
  constexpr int kWarps = kPermuteChunk / 32;
  constexpr int kChunks = kPermuteSmall / kPermuteChunk;
  __shared__ int base[kMaxExperts];  // expert offset + rows placed by earlier chunks
  __shared__ int wcnt[kWarps][kMaxExperts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int TK = T * K;
  for (int e = threadIdx.x; e < E; e += blockDim.x) base[e] = 0;
  __syncthreads();
  int ev[kChunks];
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    const int j = c * kPermuteChunk + threadIdx.x;
    ev[c] = j < TK ? load_expert(idx, j, T, K, E, status) : -1;
    if (ev[c] >= 0) atomicAdd(&base[ev[c]], 1);
  }
  __syncthreads();
  if (warp == 0) {  // totals -> exclusive offsets, in place
    int run = 0;
    for (int b = 0; b < E; b += 32) {
      const int e = b + lane;
      const int v = e < E ? base[e] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (e < E) {
        base[e] = run + incl - v;
        expert_offsets[e] = run + incl - v;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) expert_offsets[E] = run;
  }
  for (int i = threadIdx.x; i < kWarps * E; i += blockDim.x) wcnt[i / E][i % E] = 0;
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kChunks; ++c) {
    if (c * kPermuteChunk >= TK) break;  // uniform over the CTA
    const int j = c * kPermuteChunk + threadIdx.x;
    const int e = ev[c];
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank == 0) wcnt[warp][e] = __popc(peers);
    __syncthreads();
    if (j < TK) {
      const int k = j / T, t = j - k * T;
      const long long slot = static_cast<long long>(t) * K + k;
      if (e < 0) {
        slot_row[slot] = -1;
      } else {
        int before = 0;
        for (int w = 0; w < warp; ++w) before += wcnt[w][e];
        const int pos = base[e] + before + rank;
        row_token[pos] = t;
        row_slot[pos] = static_cast<int32_t>(slot);
        slot_row[slot] = pos;
        if (row_weight) row_weight[pos] = slot_weight[slot];
      }
    }
    __syncthreads();
    // advance the running bases by this chunk's counts; clear the warp counts
    for (int e2 = threadIdx.x; e2 < E; e2 += blockDim.x) {
      int add = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        add += wcnt[w][e2];
        wcnt[w][e2] = 0;
      }
      base[e2] += add;
    }
    __syncthreads();
  }
}

}  // namespace nkimoe
