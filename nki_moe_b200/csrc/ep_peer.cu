// Expert-parallel exchange over peer memory (NVLink), without a collective
// library on the data path.
//
// Every rank owns one buffer that all ranks map (CUDA IPC; no multicast
// object), laid out by ep_peer_layout():
//   step                       u32 this step's epoch (this rank's own counter)
//   disp_flag[P], res_flag[P]  u32 epoch flags (written by the peers)
//   counts[P]                  i32 rows sent by each source this step
//   recv_slots [P][Tm][K]      i32 local expert ids (-1: empty slot)
//   recv_w     [P][Tm][K]      f32 routing weights
//   recv_x     [P][Tm][H]      bf16 token rows
//   ret_y      [P][Tm][H]      bf16 partial sums
// Regions, flags and counts are indexed by the distance between the two
// ranks: region q of rank d's recv_* (and flag / count q) holds what rank
// d - q (mod P) sent; region q of rank s's ret_y (and res_flag q) holds what
// rank s + q returned.  Region 0 is the rank's own.  Source s sends token t
// to rank d once when any of t's experts lives on d (the de-duplicated
// dispatch) as row j of region q = d - s of d's buffer; d runs its local
// experts over the rows (empty slots skipped) and writes row j's weighted sum
// into row j of region q of s's ret_y; s adds its P partial sums.  Indexing by
// distance keeps the regions a receiver takes in arrival order (sources send
// to the nearest destination first) contiguous.
//
// Publication: each CTA of a sending kernel fences its peer stores at system
// scope, the last CTA to finish (a counter in local memory) publishes the
// counts and then the epoch flag with st.release.sys; a waiting rank polls its
// own flags with ld.acquire.sys under a bounded budget.  Flags hold the step's
// epoch (increasing), so they never need resetting.  Region reuse is ordered
// by the protocol itself: a rank writes into a peer's regions for step n+1
// only after it has that peer's step-n results.
#include "kernels.h"

namespace nkimoe {

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct EpPeerView {
  uint32_t* disp_flag;
  uint32_t* res_flag;
  int32_t* counts;
  int32_t* recv_slots;
  float* recv_w;
  __nv_bfloat16* recv_x;
  __nv_bfloat16* ret_y;
};

__device__ __forceinline__ EpPeerView view_of(char* base, const EpPeerLayout& L) {
  EpPeerView v;
  v.disp_flag = reinterpret_cast<uint32_t*>(base + L.disp_flag);
  v.res_flag = reinterpret_cast<uint32_t*>(base + L.res_flag);
  v.counts = reinterpret_cast<int32_t*>(base + L.counts);
  v.recv_slots = reinterpret_cast<int32_t*>(base + L.recv_slots);
  v.recv_w = reinterpret_cast<float*>(base + L.recv_w);
  v.recv_x = reinterpret_cast<__nv_bfloat16*>(base + L.recv_x);
  v.ret_y = reinterpret_cast<__nv_bfloat16*>(base + L.ret_y);
  return v;
}

// The last CTA of the grid to get here (after every CTA fenced its stores at
// system scope) returns true.  The counter is left at zero for the next use.
__device__ __forceinline__ bool last_block_done(unsigned* counter) {
  __shared__ bool last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(counter, 1u);
    last = prev == gridDim.x - 1;
    if (last) *counter = 0;
  }
  __syncthreads();
  return last;
}

// Hot-expert replicas: slot (t, k) of expert e goes to holder t mod
// counts[e] of e, i.e. to the expert slot slots[e * max_holders + t mod
// counts[e]] (slot v lives on rank v / local_slots as its local expert
// v % local_slots), which splits an expert's tokens evenly over the ranks
// that hold a copy of its weights.  An id outside [0, E), or a table entry
// outside [0, num_slots), maps to -1 (no rank takes the slot) and is flagged.
__global__ void ep_remap_kernel(const int32_t* __restrict__ idx, int T, int K, int E,
                                const int32_t* __restrict__ slots, const int32_t* __restrict__ counts,
                                int max_holders, int num_slots, int32_t* __restrict__ idx_v, int* status) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(T) * K) return;
  const int t = static_cast<int>(i / K);
  const int e = idx[i];
  int v = -1;
  if (e >= 0 && e < E) {
    const int n = counts[e];
    if (n >= 1 && n <= max_holders) v = slots[static_cast<long long>(e) * max_holders + t % n];
  }
  if (v < 0 || v >= num_slots) {
    v = -1;
    if (status) atomicOr(status, kDevErrBadIndex);
  }
  idx_v[i] = v;
}

// Source side: send row r (token row_token[r], destination d = row_slot[r] % P,
// j = r - rank_offsets[d]) of destinations [d_first, d_first + d_count) to
// region (d - src) mod P of d's buffer: the token row, its K slots as d sees
// them and their weights.  The grid walks the destinations by distance from
// src (src + 1 first, src itself last), so that while every rank sends, each
// destination is being written by one source at a time instead of all ranks
// writing to the same destination (their rows are sorted by destination rank
// alike).  One warp per pair of rows: both rows' metadata, then both rows'
// 4 KB of loads, are in flight before the stores (the stores to a peer are
// posted; the loads set the pace).  The last CTA publishes each destination's
// count and raises its dispatch flag.
__global__ void __launch_bounds__(256) ep_peer_send_kernel(
    const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ idx, const float* __restrict__ w,
    const int32_t* __restrict__ row_token, const int32_t* __restrict__ row_slot,
    const int32_t* __restrict__ rank_offsets, int H, int K, int P, int El, int Tm, int src, int d_first, int d_count,
    EpPeerPtrs peers, EpPeerLayout L, unsigned* counter, const uint32_t* epoch_p) {
  constexpr int kRowsPerWarp = 2;
  // destinations in walking order and where each starts in the walk
  __shared__ int s_dest[kMaxPeers + 1], s_start[kMaxPeers + 1];
  if (threadIdx.x == 0) {
    int n = 0, o = 0;
    for (int q = 1; q <= P; ++q) {
      const int d = (src + q) % P;
      if (d < d_first || d >= d_first + d_count) continue;
      s_dest[n] = d;
      s_start[n] = o;
      o += rank_offsets[d + 1] - rank_offsets[d];
      ++n;
    }
    s_start[n] = o;
    s_dest[n] = n;  // number of destinations walked
  }
  __syncthreads();
  const int nd = s_dest[d_count];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long rows = s_start[nd];
  const int chunks = H >> 3;
  for (long long i0 = (static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kRowsPerWarp;
       i0 < rows; i0 += nw * kRowsPerWarp) {
    int t[kRowsPerWarp], d[kRowsPerWarp];
    long long dst_row[kRowsPerWarp];
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q) {
      const long long i = i0 + q < rows ? i0 + q : i0;
      int k = 0;
      while (k + 1 < nd && s_start[k + 1] <= i) ++k;
      d[q] = s_dest[k];
      const long long jrow = i - s_start[k];
      const long long r = rank_offsets[d[q]] + jrow;
      t[q] = row_token[r];
      const int region = (d[q] - src + P) % P;
      dst_row[q] = static_cast<long long>(region) * Tm + jrow;
    }
    for (int c0 = lane; c0 < chunks; c0 += 256) {
      uint4 v[kRowsPerWarp][8];
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) {
        const uint4* s4 = reinterpret_cast<const uint4*>(x + static_cast<long long>(t[q]) * H);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (c0 + 32 * u < chunks) v[q][u] = s4[c0 + 32 * u];
      }
#pragma unroll
      for (int q = 0; q < kRowsPerWarp; ++q) {
        if (i0 + q >= rows) break;
        uint4* d4 = reinterpret_cast<uint4*>(view_of(peers.base[d[q]], L).recv_x + dst_row[q] * H);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (c0 + 32 * u < chunks) d4[c0 + 32 * u] = v[q][u];
      }
    }
#pragma unroll
    for (int q = 0; q < kRowsPerWarp; ++q) {
      if (i0 + q >= rows || lane >= K) continue;
      const EpPeerView pv = view_of(peers.base[d[q]], L);
      const int e = idx[static_cast<long long>(t[q]) * K + lane];
      const bool mine = e >= d[q] * El && e < (d[q] + 1) * El;
      pv.recv_slots[dst_row[q] * K + lane] = mine ? e - d[q] * El : -1;
      pv.recv_w[dst_row[q] * K + lane] = mine ? w[static_cast<long long>(t[q]) * K + lane] : 0.f;
    }
  }
  if (last_block_done(counter) && threadIdx.x < d_count) {
    const int d = d_first + threadIdx.x;
    const int region = (d - src + P) % P;
    const EpPeerView pv = view_of(peers.base[d], L);
    pv.counts[region] = rank_offsets[d + 1] - rank_offsets[d];
    __threadfence_system();
    st_release_sys(pv.disp_flag + region, *epoch_p);
  }
}

// Source-side bookkeeping: slot_out[t * P + d] = the row of ret_y that will
// hold the partial sum of token t from rank d (region (d - src) mod P, at the
// row t was sent to; region 0 at row t when self_direct), -1 when t has no
// expert on d; and with self_idx, t's slots as this rank sees them.
__global__ void ep_peer_local_kernel(const int32_t* __restrict__ idx, const float* __restrict__ w,
                                     const int32_t* __restrict__ slot_in, const int32_t* __restrict__ rank_offsets,
                                     int T, int K, int P, int El, int Tm, int src, int self_direct,
                                     int32_t* __restrict__ slot_out, int32_t* __restrict__ self_idx,
                                     float* __restrict__ self_w) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  const long long i0 = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (long long i = i0; i < static_cast<long long>(T) * P; i += stride) {
    const int d = static_cast<int>(i % P);
    const int sr = slot_in[i];
    const int region = (d - src + P) % P;
    int row = -1;
    if (sr >= 0) row = (self_direct && d == src) ? static_cast<int>(i / P) : region * Tm + (sr - rank_offsets[d]);
    slot_out[i] = row;
  }
  if (self_idx) {
    for (long long i = i0; i < static_cast<long long>(T) * K; i += stride) {
      const int e = idx[i];
      const bool mine = e >= src * El && e < (src + 1) * El;
      self_idx[i] = mine ? e - src * El : -1;
      self_w[i] = mine ? w[i] : 0.f;
    }
  }
}

// Poll flags[0 .. n) until each holds the step's epoch, for at most `budget`
// SM clock cycles; a flag still behind then sets the timeout bit of the status
// word and the kernel returns.  One warp.
__global__ void ep_peer_wait_kernel(const uint32_t* flags, int n, const uint32_t* epoch_p, int* status,
                                    long long budget) {
  const uint32_t epoch = *epoch_p;
  const int lane = threadIdx.x;
  bool ok = true;
  if (lane < n) {
    const long long t0 = clock64();
    while (static_cast<int>(ld_acquire_sys(flags + lane) - epoch) < 0) {
      if (clock64() - t0 > budget) {
        ok = false;
        break;
      }
      __nanosleep(200);
    }
  }
  if (!ok) atomicOr(status, kDevErrTimeout);
}

// Receiver: rows past each source's count get empty slots (the region holds
// whatever an earlier step left there).  `slots` starts at region q0.
__global__ void ep_peer_mask_kernel(int32_t* __restrict__ slots, const int32_t* __restrict__ counts, int q0, int nq,
                                    int Tm, int K) {
  const long long n = static_cast<long long>(nq) * Tm * K;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / K;
    const int q = static_cast<int>(row / Tm);
    const long long j = row - static_cast<long long>(q) * Tm;
    if (j >= counts[q0 + q]) slots[i] = -1;
  }
}

// Receiver: the routing-weighted sum of row r's K expert outputs (fp32, k
// ascending, as combine_kernel), stored straight into the source's ret_y: row
// r is row j = r % Tm of region q = q0 + r / Tm, from source s = me - q, and
// its sum goes to row j of region q of s's ret_y.  Rows without a local
// expert are skipped.  One warp per row: its K output-row indices come in one
// load, then each present slot's whole 4 KB row is loaded (8 x 16 bytes per
// lane in flight) and added; the sum leaves as 4 KB of contiguous stores.  The
// last CTA raises the result flags of the regions' sources.
__global__ void __launch_bounds__(256) ep_peer_combine_kernel(const __nv_bfloat16* __restrict__ y,
                                                              const int32_t* __restrict__ slot_row, int q0, int nq,
                                                              int K, int H, int Tm, int me, EpPeerPtrs peers,
                                                              EpPeerLayout L, int P, unsigned* counter,
                                                              const uint32_t* epoch_p,
                                                              __nv_bfloat16* __restrict__ local_ret) {
  const int lane = threadIdx.x & 31;
  const int chunks = H >> 3;
  const long long rows = static_cast<long long>(nq) * Tm;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  // when the rows include region 0 (this rank's own, no NVLink), it is taken
  // last, so the remote regions' stores start at once
  const long long shift = (q0 == 0 && nq > 1) ? Tm : 0;
  for (long long i = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); i < rows;
       i += nw) {
    const long long r = i + shift < rows ? i + shift : i + shift - rows;
    const int my_yr = lane < K ? slot_row[r * K + lane] : -1;
    const unsigned present = __ballot_sync(0xffffffffu, my_yr >= 0);
    if (present == 0u) continue;
    const int q = q0 + static_cast<int>(r / Tm);
    const long long j = r % Tm;
    const int s = (me - q + P) % P;
    __nv_bfloat16* ret = local_ret ? local_ret : view_of(peers.base[s], L).ret_y;
    uint4* dst = reinterpret_cast<uint4*>(ret + (static_cast<long long>(q) * Tm + j) * H);
    for (int c0 = lane; c0 < chunks; c0 += 256) {
      float acc[8][8] = {};
      for (unsigned m = present; m != 0u; m &= m - 1u) {  // slots in ascending k
        const int yr = __shfl_sync(0xffffffffu, my_yr, __ffs(m) - 1);
        const uint4* src = reinterpret_cast<const uint4*>(y + static_cast<long long>(yr) * H);
        uint4 u[8];
#pragma unroll
        for (int qq = 0; qq < 8; ++qq)
          if (c0 + 32 * qq < chunks) u[qq] = __ldcs(src + c0 + 32 * qq);
#pragma unroll
        for (int qq = 0; qq < 8; ++qq) {
          if (c0 + 32 * qq >= chunks) break;
          const float2 a = unpack_bf16x2(u[qq].x), b = unpack_bf16x2(u[qq].y);
          const float2 cc = unpack_bf16x2(u[qq].z), dd = unpack_bf16x2(u[qq].w);
          acc[qq][0] += a.x;
          acc[qq][1] += a.y;
          acc[qq][2] += b.x;
          acc[qq][3] += b.y;
          acc[qq][4] += cc.x;
          acc[qq][5] += cc.y;
          acc[qq][6] += dd.x;
          acc[qq][7] += dd.y;
        }
      }
#pragma unroll
      for (int qq = 0; qq < 8; ++qq) {
        if (c0 + 32 * qq >= chunks) break;
        uint4 o;
        o.x = pack_bf16x2(acc[qq][0], acc[qq][1]);
        o.y = pack_bf16x2(acc[qq][2], acc[qq][3]);
        o.z = pack_bf16x2(acc[qq][4], acc[qq][5]);
        o.w = pack_bf16x2(acc[qq][6], acc[qq][7]);
        dst[c0 + 32 * qq] = o;
      }
    }
  }
  if (local_ret) return;
  if (last_block_done(counter) && threadIdx.x < nq) {
    const int q = q0 + threadIdx.x;
    const EpPeerView pv = view_of(peers.base[(me - q + P) % P], L);
    st_release_sys(pv.res_flag + q, *epoch_p);
  }
}

// Copy-engine send, local half: rows of the destinations d != src to this
// rank's staging regions (row j of destination d at d * Tm + j), the rows'
// slots as d sees them and their weights; stage_counts[d] = d's row count.
__global__ void __launch_bounds__(256) ep_peer_stage_kernel(
    const __nv_bfloat16* __restrict__ x, const int32_t* __restrict__ idx, const float* __restrict__ w,
    const int32_t* __restrict__ row_token, const int32_t* __restrict__ row_slot,
    const int32_t* __restrict__ rank_offsets, int H, int K, int P, int El, int Tm, int src,
    __nv_bfloat16* __restrict__ stage_x, int32_t* __restrict__ stage_slots, float* __restrict__ stage_w,
    int32_t* __restrict__ stage_counts) {
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const long long rows = rank_offsets[P];
  const int chunks = H >> 3;
  if (blockIdx.x == 0 && threadIdx.x < P) stage_counts[threadIdx.x] = rank_offsets[threadIdx.x + 1] - rank_offsets[threadIdx.x];
  for (long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += nw) {
    const int d = row_slot[r] % P;
    if (d == src) continue;  // the own tokens' share is computed from x directly
    const int t = row_token[r];
    const long long dst_row = static_cast<long long>(d) * Tm + (r - rank_offsets[d]);
    const uint4* s4 = reinterpret_cast<const uint4*>(x + static_cast<long long>(t) * H);
    uint4* d4 = reinterpret_cast<uint4*>(stage_x + dst_row * H);
    for (int c0 = lane; c0 < chunks; c0 += 256) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + 32 * u < chunks) v[u] = s4[c0 + 32 * u];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (c0 + 32 * u < chunks) d4[c0 + 32 * u] = v[u];
    }
    if (lane < K) {
      const int e = idx[static_cast<long long>(t) * K + lane];
      const bool mine = e >= d * El && e < (d + 1) * El;
      stage_slots[dst_row * K + lane] = mine ? e - d * El : -1;
      stage_w[dst_row * K + lane] = mine ? w[static_cast<long long>(t) * K + lane] : 0.f;
    }
  }
}

__global__ void ep_peer_publish_kernel(int32_t* count_dst, const int32_t* count_src, uint32_t* flag,
                                       const uint32_t* epoch_p) {
  if (count_src) *count_dst = *count_src;
  __threadfence_system();
  st_release_sys(flag, *epoch_p);
}

// The step's epoch in this rank's own buffer: `value` when nonzero (the
// caller counts steps), otherwise the stored epoch + 1 (the device counts, so
// that a captured CUDA graph advances it on every replay).
__global__ void ep_peer_step_kernel(uint32_t* step, uint32_t value) {
  *step = value != 0u ? value : *step + 1u;
}

unsigned grid_cap(long long work, int threads) {
  const long long b = (work + threads - 1) / threads;
  const long long cap = static_cast<long long>(device_sm_count()) * 8;
  return static_cast<unsigned>(b < 1 ? 1 : (b > cap ? cap : b));
}

size_t r256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

}  // namespace

EpPeerLayout ep_peer_layout(long long P, long long Tm, long long H, long long K) {
  EpPeerLayout L{};
  size_t o = 0;
  L.step = o;
  o += 256;
  L.disp_flag = o;
  o += r256(sizeof(uint32_t) * P);
  L.res_flag = o;
  o += r256(sizeof(uint32_t) * P);
  L.counts = o;
  o += r256(sizeof(int32_t) * P);
  L.recv_slots = o;
  o += r256(sizeof(int32_t) * P * Tm * K);
  L.recv_w = o;
  o += r256(sizeof(float) * P * Tm * K);
  L.recv_x = o;
  o += r256(sizeof(uint16_t) * P * Tm * H);
  L.ret_y = o;
  o += r256(sizeof(uint16_t) * P * Tm * H);
  L.total = o;
  return L;
}

cudaError_t ep_peer_send_launch(const __nv_bfloat16* x, const int32_t* idx, const float* w, const int32_t* row_token,
                                const int32_t* row_slot, const int32_t* rank_offsets, int T, int H, int K, int P,
                                int El, int Tm, int src, int d_first, int d_count, const EpPeerPtrs& peers,
                                const EpPeerLayout& L, unsigned* counter, const uint32_t* epoch_p, int max_ctas,
                                cudaStream_t s) {
  if (d_first < 0 || d_count < 1 || d_first + d_count > P || d_count > 256) return cudaErrorInvalidValue;
  // one warp per two send rows (at most T rows per destination); at least one
  // CTA so that the flags are raised even when nothing is sent
  unsigned grid = grid_cap(static_cast<long long>(T) * d_count * 16, 256);
  if (max_ctas > 0 && grid > static_cast<unsigned>(max_ctas)) grid = static_cast<unsigned>(max_ctas);
  ep_peer_send_kernel<<<grid, 256, 0, s>>>(x, idx, w, row_token, row_slot, rank_offsets, H, K, P, El, Tm, src,
                                           d_first, d_count, peers, L, counter, epoch_p);
  return cudaGetLastError();
}

cudaError_t ep_peer_local_launch(const int32_t* idx, const float* w, const int32_t* slot_in,
                                 const int32_t* rank_offsets, int T, int K, int P, int El, int Tm, int src,
                                 bool self_direct, int32_t* slot_out, int32_t* self_idx, float* self_w, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  const long long work = static_cast<long long>(T) * (P > K ? P : K);
  ep_peer_local_kernel<<<grid_cap(work, 256), 256, 0, s>>>(idx, w, slot_in, rank_offsets, T, K, P, El, Tm, src,
                                                           self_direct ? 1 : 0, slot_out, self_idx, self_w);
  return cudaGetLastError();
}

cudaError_t ep_peer_step_launch(uint32_t* step, uint32_t value, cudaStream_t s) {
  ep_peer_step_kernel<<<1, 1, 0, s>>>(step, value);
  return cudaGetLastError();
}

cudaError_t ep_remap_launch(const int32_t* idx, int T, int K, int E, const int32_t* slots, const int32_t* counts,
                            int max_holders, int num_slots, int32_t* idx_v, int* status, cudaStream_t s) {
  if (T == 0) return cudaSuccess;
  if (max_holders < 1) return cudaErrorInvalidValue;
  const long long n = static_cast<long long>(T) * K;
  ep_remap_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(idx, T, K, E, slots, counts, max_holders,
                                                                         num_slots, idx_v, status);
  return cudaGetLastError();
}

cudaError_t ep_peer_wait_launch(const uint32_t* flags, int n, const uint32_t* epoch_p, int* status,
                                long long budget_cycles, cudaStream_t s) {
  if (n < 1 || n > 32) return cudaErrorInvalidValue;
  ep_peer_wait_kernel<<<1, 32, 0, s>>>(flags, n, epoch_p, status, budget_cycles);
  return cudaGetLastError();
}

cudaError_t ep_peer_mask_launch(int32_t* slots, const int32_t* counts, int q0, int nq, int Tm, int K, cudaStream_t s) {
  ep_peer_mask_kernel<<<grid_cap(static_cast<long long>(nq) * Tm * K, 256), 256, 0, s>>>(slots, counts, q0, nq, Tm,
                                                                                        K);
  return cudaGetLastError();
}

cudaError_t ep_peer_combine_launch(const __nv_bfloat16* y, const int32_t* slot_row, int q0, int nq, int K, int H,
                                   int Tm, int me, const EpPeerPtrs& peers, const EpPeerLayout& L, int P,
                                   unsigned* counter, const uint32_t* epoch_p, int max_ctas, cudaStream_t s,
                                   __nv_bfloat16* local_ret) {
  if (nq < 1 || q0 < 0 || q0 + nq > P) return cudaErrorInvalidValue;
  unsigned grid = grid_cap(static_cast<long long>(nq) * Tm * 32, 256);  // one warp per row
  if (max_ctas > 0 && grid > static_cast<unsigned>(max_ctas)) grid = static_cast<unsigned>(max_ctas);
  ep_peer_combine_kernel<<<grid, 256, 0, s>>>(y, slot_row, q0, nq, K, H, Tm, me, peers, L, P, counter, epoch_p,
                                              local_ret);
  return cudaGetLastError();
}

cudaError_t ep_peer_stage_launch(const __nv_bfloat16* x, const int32_t* idx, const float* w, const int32_t* row_token,
                                 const int32_t* row_slot, const int32_t* rank_offsets, int T, int H, int K, int P,
                                 int El, int Tm, int src, __nv_bfloat16* stage_x, int32_t* stage_slots,
                                 float* stage_w, int32_t* stage_counts, cudaStream_t s) {
  if (P > 256) return cudaErrorInvalidValue;
  const unsigned grid = grid_cap(static_cast<long long>(T) * P * 32, 256);  // one warp per row
  ep_peer_stage_kernel<<<grid, 256, 0, s>>>(x, idx, w, row_token, row_slot, rank_offsets, H, K, P, El, Tm, src,
                                            stage_x, stage_slots, stage_w, stage_counts);
  return cudaGetLastError();
}

cudaError_t ep_peer_publish_launch(int32_t* count_dst, const int32_t* count_src, uint32_t* flag,
                                   const uint32_t* epoch_p, cudaStream_t s) {
  ep_peer_publish_kernel<<<1, 1, 0, s>>>(count_dst, count_src, flag, epoch_p);
  return cudaGetLastError();
}

}  // namespace nkimoe
