// K4/K5: grouped expert GEMMs on the 5th-generation tensor cores.
//
// Problem: for every expert e, rows [off[e], off[e+1]) of a permuted
// activation matrix A (K-major, bf16) are multiplied by that expert's packed
// weight W[e] (N x K, K-major, bf16):  C_e = A_e . W[e]^T, fp32 accumulate.
// Used twice per MoE block (nki_moe_integrated.py:154-161):
//   GEMM-1: A = gathered tokens [R, H], W13[e] = [2I, H] -> SwiGLU epilogue -> h [R, I]
//   GEMM-2: A = h [R, I],               W2[e]  = [H, I]  -> routing-weight epilogue -> Y [R, H]
//
// Two tile schedules over the same machinery:
//   rows    (prefill): tile = 128 rows x BN features; A is the MMA's A operand.
//   weights (decode):  tile = 128 features x BT rows ("swap AB"); the weight
//                      block is the MMA's A operand so a handful of tokens per
//                      expert still fills the 128-wide M dimension, and every
//                      CTA streams whole weight blocks at HBM speed.
//
// Structure (persistent, one CTA per SM, 192 threads):
//   warp 0: TMA producer     — fills a STAGES-deep ring of smem stages
//   warp 1: MMA issuer       — tcgen05.mma (M=128, K=16 per instruction) into
//                              one of two TMEM accumulators; tcgen05.commit
//                              releases smem stages and publishes accumulators
//   warps 2-5: epilogue      — tcgen05.ld, fused SwiGLU / scale, bf16 stores
// Tiles are enumerated on the device from expert_offsets (no host sync):
// expert-major, then feature block, then row block, so concurrently running
// CTAs share weight panels through L2.
#include <algorithm>
#include <map>
#include <mutex>
#include <set>
#include <utility>

#include "kernels.h"

namespace nkimoe {

namespace {

constexpr int kThreads = 192;
constexpr int BM = 128;  // MMA M (rows of the A operand per tile)
constexpr int BK = 64;   // bf16 elements per 128-byte swizzled row
constexpr int UK = 16;   // K per tcgen05.mma kind::f16

struct SharedCtl {
  uint64_t full[16];
  uint64_t empty[16];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int seg[kMaxExperts + 1];         // first row of each expert's rows in this launch
  int seg_end[kMaxExperts];         // one past its last row
  int tile_start[kMaxExperts + 1];  // first tile of each expert
};

// Row split between the SM-pair kernel and the 1-SM kernel (row_split 1 / 2
// in GroupedGemmParams): the pair takes each expert's whole blocks of this
// many rows, the 1-SM kernel the rows past them.
constexpr int kSplitRows = 256;

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~static_cast<uintptr_t>(1023));
}

// Warp-wide: lane 0 waits, the result is broadcast (keeps the warp converged
// for the .sync.aligned tcgen05 instructions that follow).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, SharedCtl& ctl, int* status) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, &ctl.abort_flag, status);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// Short bounded wait used only while tearing down after an abort.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles / 8) break;
  }
}

// Per-expert tile table in smem.  tiles(e) = ceil(rows_e / rows_per_tile) * feat_tiles.
__device__ void build_tile_table(SharedCtl& ctl, const int32_t* offs, int dense_rows, int E, int rows_per_tile,
                                 int feat_tiles, int row_split = 0) {
  const int lane = threadIdx.x & 31;
  int run = 0;
  for (int b = 0; b < E; b += 32) {
    const int e = b + lane;
    int cnt = 0, s0 = 0;
    if (e < E) {
      s0 = offs ? offs[e] : e * dense_rows;
      cnt = offs ? offs[e + 1] - s0 : dense_rows;
      if (row_split == 1) {
        cnt -= cnt % kSplitRows;  // whole blocks only
      } else if (row_split == 2) {
        s0 += cnt - cnt % kSplitRows;  // the rows past the whole blocks
        cnt %= kSplitRows;
      }
    }
    const int tiles = ((cnt + rows_per_tile - 1) / rows_per_tile) * feat_tiles;
    int incl = tiles;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (e < E) {
      ctl.tile_start[e] = run + incl - tiles;
      ctl.seg[e] = s0;
      ctl.seg_end[e] = s0 + cnt;
    }
    run += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    ctl.tile_start[E] = run;
    ctl.seg[E] = offs ? offs[E] : E * dense_rows;
  }
}

struct TileCoord {
  int e;       // expert
  int rblk;    // row block within the expert
  int fblk;    // feature block within the expert
};

__device__ __forceinline__ TileCoord decode_tile(const SharedCtl& ctl, int E, int tile, int rows_per_tile,
                                                 int feat_tiles) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ctl.tile_start[mid] <= tile) lo = mid;
    else hi = mid - 1;
  }
  const int local = tile - ctl.tile_start[lo];
  const int rtiles = (ctl.tile_start[lo + 1] - ctl.tile_start[lo]) / feat_tiles;
  TileCoord c;
  c.e = lo;
  c.fblk = local / rtiles;
  c.rblk = local % rtiles;
  (void)rows_per_tile;
  return c;
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float (&v)[N]) {
  static_assert(N % 16 == 0, "column count");
  if constexpr (N % 32 == 0) {
#pragma unroll
    for (int c = 0; c < N; c += 32) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + c, r);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) v[c + j] = __uint_as_float(r[j]);
    }
  } else {
    uint32_t r[16];
    tmem_ld_32x32b_x16(taddr, r);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
    u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
    u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
    u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    d[q] = u;
  }
}

// Store 32 bf16 values of this lane's output row (columns [col, col + 32))
// through the warp's 32 x 32 staging tile: each lane writes its row, then lane
// l stores 16 bytes of row l / 4 + 8 i, so one store instruction covers 8 rows
// x 64 contiguous bytes (whole sectors) instead of 32 rows x 16 bytes.
__device__ __forceinline__ void store_row32_staged(__nv_bfloat16 (*st)[40], __nv_bfloat16* out, long long ld,
                                                   long long orow, bool valid, long long col, const float (&v)[32],
                                                   int lane) {
  uint4* srow = reinterpret_cast<uint4*>(&st[lane][0]);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
    u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
    u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
    u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    srow[q] = u;
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = (lane >> 2) + 8 * i;
    const long long o = __shfl_sync(0xffffffffu, orow, rr);
    const bool vr = __shfl_sync(0xffffffffu, valid ? 1 : 0, rr) != 0;
    if (vr)
      *reinterpret_cast<uint4*>(out + o * ld + col + (lane & 3) * 8) =
          *reinterpret_cast<const uint4*>(&st[rr][(lane & 3) * 8]);
  }
  __syncwarp();
}

// Epilogue of a rows-schedule tile for one thread = one output row: reads the
// row's BN accumulator columns from tensor memory (all lanes of the warp must
// call it: tcgen05.ld is warp-collective) and stores them per p.epilogue
// (bf16 outputs through the warp's staging tile `st`).
template <int BN>
__device__ __forceinline__ void rows_epilogue(const GroupedGemmParams& p, uint32_t tbase, int fblk, long long orow,
                                              bool valid, float scale, __nv_bfloat16 (*st)[40], int lane) {
  if (p.epilogue == kEpiSwiGLU) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
    for (int blk = 0; blk < BN / 128; ++blk) {
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float g[32], u[32];
        tmem_ld_cols<32>(tbase + blk * 128 + half * 32, g);
        tmem_ld_cols<32>(tbase + blk * 128 + 64 + half * 32, u);
        float h[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) h[j] = silu_f(g[j]) * u[j];
        const long long col = static_cast<long long>(fblk) * (BN / 2) + blk * 64 + half * 32;
        if (p.stage_stores & 1) store_row32_staged(st, out, p.out_ld, orow, valid, col, h, lane);
        else if (valid) store_bf16x32(out + orow * p.out_ld + col, h);
      }
    }
  } else if (p.epilogue == kEpiScaleBf16 || p.epilogue == kEpiStoreBf16) {
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld_cols<32>(tbase + c, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] *= scale;
      const long long col = static_cast<long long>(fblk) * BN + c;
      if (p.stage_stores & 2) store_row32_staged(st, out, p.out_ld, orow, valid, col, v, lane);
      else if (valid) store_bf16x32(out + orow * p.out_ld + col, v);
    }
  } else {  // kEpiStoreF32: two 16-column passes through the staging tile (64 B per row)
    float* out = static_cast<float*>(p.out);
    float(*sf)[20] = reinterpret_cast<float(*)[20]>(st);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld_cols<32>(tbase + c, v);
      const long long col0 = static_cast<long long>(fblk) * BN + c;
      if (p.col_bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += p.col_bias[col0 + j];
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float4* srow = reinterpret_cast<float4*>(&sf[lane][0]);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          srow[q] = make_float4(v[hf * 16 + 4 * q], v[hf * 16 + 4 * q + 1], v[hf * 16 + 4 * q + 2],
                                v[hf * 16 + 4 * q + 3]);
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = (lane >> 2) + 8 * i;
          const long long o = __shfl_sync(0xffffffffu, orow, rr);
          const bool vr = __shfl_sync(0xffffffffu, valid ? 1 : 0, rr) != 0;
          if (vr)
            *reinterpret_cast<float4*>(out + o * p.out_ld + col0 + hf * 16 + (lane & 3) * 4) =
                *reinterpret_cast<const float4*>(&sf[rr][(lane & 3) * 4]);
        }
        __syncwarp();
      }
    }
  }
}

// Producer-warp gather of one 64-element K block of NR activation rows into a
// stage laid out exactly as a 128-byte-swizzled TMA box (16-byte chunk c of
// row i at chunk c ^ (i % 8) of the row's 128 bytes).  src_row[j] is the
// source row of tile row lane + 32 j (-1: zero fill).
template <int NR>
__device__ __forceinline__ void gather_k_block(uint32_t sdst, const __nv_bfloat16* a, long long ld, int kcol,
                                               const int (&src_row)[(NR + 31) / 32], int lane) {
#pragma unroll
  for (int j = 0; j < (NR + 31) / 32; ++j) {
    const int i = lane + 32 * j;
    if (NR % 32 == 0 || i < NR) {
      const int sr = src_row[j];
      const __nv_bfloat16* src = a + (sr >= 0 ? static_cast<long long>(sr) * ld : 0) + kcol;
      const uint32_t nbytes = sr >= 0 ? 16u : 0u;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        cp_async_16(sdst + i * 128 + ((c ^ (i & 7)) << 4), src + c * 8, nbytes);
    }
  }
}

// ============================================================ rows schedule
// Tile: 128 activation rows x BN packed features.  A = activations (box 64 x
// 128), B = weights (box 64 x BN), D[row][feature] in TMEM lanes x columns.
template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_rows_kernel(const __grid_constant__ CUtensorMap tmap_act, const __grid_constant__ CUtensorMap tmap_w,
                             const GroupedGemmParams p) {
  constexpr uint32_t A_BYTES = BM * BK * 2;
  constexpr uint32_t B_BYTES = BN * BK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(STAGES <= 16, "stages");

  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedCtl ctl;
  __shared__ __align__(16) __nv_bfloat16 stg[4][32][40];  // per epilogue warp: output staging
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.num_experts;
  const int feat_tiles = p.n / BN;

  const bool gather_a = p.a_row_map != nullptr;
  const bool gather_cp = gather_a && !p.tma_gather4;  // rows written by cp.async (generic proxy)
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl.full[s], gather_cp ? 1 + 32 : 1);  // + one cp.async arrival per producer lane
      mbar_init(&ctl.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl.acc_full[a], 1);
      mbar_init(&ctl.acc_empty[a], 4 * 32);
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_act);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) tmem_alloc(&ctl.tmem_base, TMEM_COLS);
  if (warp == 2) build_tile_table(ctl, p.expert_offsets, p.dense_rows, E, BM, feat_tiles, p.row_split);
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total_tiles = ctl.tile_start[E];

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    // TMA mode: lane 0 alone runs the loop (no per-stage warp collectives);
    // gather mode: the whole warp issues the cp.async row gathers.
    if (gather_a || lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_phase_mask = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x) {
        const TileCoord tc = decode_tile(ctl, E, tile, BM, feat_tiles);
        const int row0 = ctl.seg[tc.e] + tc.rblk * BM;
        const int arow0 = p.shared_a ? tc.rblk * BM : row0;
        const int wrow0 = (p.weight_mod ? tc.e % p.weight_mod : tc.e) * p.n + tc.fblk * BN;
        // cp.async gather: tile row lane + 32 j; TMA gather4: tile rows 4 lane + j
        // (rows past the segment end re-read the tile's first row; their
        // accumulator rows are never stored)
        int src_row[BM / 32];
        if (gather_a) {
          const int seg_end = ctl.seg_end[tc.e];
          const int first = p.a_row_map[row0];
#pragma unroll
          for (int j = 0; j < BM / 32; ++j) {
            const int r = gather_cp ? row0 + lane + 32 * j : row0 + 4 * lane + j;
            src_row[j] = r < seg_end ? p.a_row_map[r] : (gather_cp ? -1 : first);
          }
        }
        int ka = 0;  // activation K coordinate (wraps at k_blocks_a blocks)
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (gather_a) {
            if (!warp_wait(&ctl.empty[stage], phase ^ 1u, ctl, p.status)) {
              ok = false;
              break;
            }
            if (lane == 0) {
              mbar_arrive_expect_tx(&ctl.full[stage], gather_cp ? B_BYTES : STAGE_BYTES);
              tma_load_2d(sb + stage * B_BYTES, &tmap_w, &ctl.full[stage], kb * BK, wrow0);
            }
            if (gather_cp) {
              gather_k_block<BM>(smem_u32(sa + stage * A_BYTES), p.a_ptr, p.a_ld, ka, src_row, lane);
              cp_async_mbar_arrive(&ctl.full[stage]);
            } else {  // 32 lanes x 4 rows x 128 bytes = the 128-row A stage
              __syncwarp();
              tma_gather4_2d(sa + stage * A_BYTES + lane * 512, &tmap_act, &ctl.full[stage], ka, src_row[0],
                             src_row[1], src_row[2], src_row[3]);
            }
          } else {
            if (!mbar_wait(&ctl.empty[stage], phase ^ 1u, &ctl.abort_flag, p.status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&ctl.full[stage], STAGE_BYTES);
            tma_load_2d(sa + stage * A_BYTES, &tmap_act, &ctl.full[stage], ka, arow0);
            tma_load_2d(sb + stage * B_BYTES, &tmap_w, &ctl.full[stage], kb * BK, wrow0);
            // At the start of a tile, pull the first p.prefetch K blocks of this
            // CTA's next tile into L2: its weight panel then comes from L2, not
            // DRAM, when the ring reaches it (hides the tile-boundary latency).
            if (kb == 0 && p.prefetch && tile + static_cast<int>(gridDim.x) < total_tiles) {
              const TileCoord nc = decode_tile(ctl, E, tile + gridDim.x, BM, feat_tiles);
              const int pw = (p.weight_mod ? nc.e % p.weight_mod : nc.e) * p.n + nc.fblk * BN;
              const int pa = p.shared_a ? nc.rblk * BM : ctl.seg[nc.e] + nc.rblk * BM;
              const int npf = min(p.prefetch, p.k_blocks);
              for (int pk = 0; pk < npf; ++pk) {
                tma_prefetch_2d(&tmap_act, (pk % p.k_blocks_a) * BK, pa);
                tma_prefetch_2d(&tmap_w, pk * BK, pw);
              }
            }
          }
          ka += BK;
          if (ka == p.k_blocks_a * BK) ka = 0;
          issued_mask |= 1u << stage;
          last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && lane == 0) {  // let copies in flight land before the CTA exits
        for (int s = 0; s < STAGES; ++s)
          if ((issued_mask >> s) & 1u) drain_wait(&ctl.full[s], (last_phase_mask >> s) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    // One thread issues every MMA and commit; its loop has no warp
    // collectives.  The mbarrier wait orders the TMA-written stage before the
    // MMAs that read it; tcgen05 fences are needed only at the TMEM hand-offs.
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      int t_local = 0;
      for (int tile = blockIdx.x; ok && tile < total_tiles; tile += gridDim.x, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t acc_phase = (t_local >> 1) & 1;
        if (!mbar_wait(&ctl.acc_empty[acc], acc_phase ^ 1u, &ctl.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ctl.full[stage], phase, &ctl.abort_flag, p.status)) {
            ok = false;
            break;
          }
          if (gather_cp) fence_proxy_async_shared();  // cp.async-written A -> tensor-core reads
          // K step of 16 bf16 = 32 bytes = 2 in the descriptor's address field
          const uint64_t da = umma_desc_sw128(smem_u32(sa + stage * A_BYTES));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / UK; ++kk)
            umma_bf16(d_tmem, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&ctl.empty[stage]);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&ctl.acc_full[acc]);
      }
      if (!ok && issued) {  // wait for issued MMAs before TMEM is released
        umma_commit(&ctl.drain);
        drain_wait(&ctl.drain, 0);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row_in_tile = quarter * 32 + lane;
    int t_local = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++t_local) {
      const TileCoord tc = decode_tile(ctl, E, tile, BM, feat_tiles);
      const int acc = t_local & 1;
      const uint32_t acc_phase = (t_local >> 1) & 1;
      const int seg_end = ctl.seg_end[tc.e];
      const int r = ctl.seg[tc.e] + tc.rblk * BM + row_in_tile;
      const bool valid = r < seg_end;
      // per-row loads issued before the accumulator wait so their latency overlaps it
      const long long orow = valid ? (p.out_row_map ? p.out_row_map[r] : r) : 0;
      float scale = 1.f;
      if (p.epilogue == kEpiScaleBf16 && valid) scale = p.row_weight ? p.row_weight[r] : p.slot_weight[p.row_slot[r]];
      if (!warp_wait(&ctl.acc_full[acc], acc_phase, ctl, p.status)) break;
      tcgen05_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;

      rows_epilogue<BN>(p, tbase, tc.fblk, orow, valid, scale, stg[quarter], lane);
      tcgen05_fence_before();
      mbar_arrive(&ctl.acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tcgen05_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ============================================================ rows schedule, SM pair
// Tile: 256 activation rows x BN features computed by a 2-CTA cluster with
// tcgen05.mma.cta_group::2 (M = 256).  CTA r of the pair loads activation rows
// [128 r, 128 r + 128) and weight rows [r BN/2, (r + 1) BN/2) of the tile into
// its own shared memory, so each SM fetches half of the B operand of a
// 256 x BN tile: 64 B per cycle per SM from L2 at full MMA rate instead of
// 96 B for a 1-SM 128 x 256 tile.  Both CTAs' loads complete on the even
// (leader) CTA's stage barrier (cta_group::2 form of the tiled load; each CTA
// fetches only its own box), which the leader arms with both halves' bytes;
// the leader issues the MMAs, its tcgen05.commit arrives on the stage and
// accumulator barriers of both CTAs, and the odd CTA's epilogue warps arrive
// remotely on the leader's "accumulator free" barrier.
template <int BN, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_rows2_kernel(const __grid_constant__ CUtensorMap tmap_act, const __grid_constant__ CUtensorMap tmap_w,
                              const GroupedGemmParams p) {
  constexpr int BM2 = 2 * BM;                       // rows per pair tile
  constexpr uint32_t A_BYTES = BM * BK * 2;         // this CTA's 128 rows
  constexpr uint32_t B_BYTES = (BN / 2) * BK * 2;   // this CTA's BN/2 weight rows
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(STAGES <= 16, "stages");

  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedCtl ctl;
  __shared__ __align__(16) __nv_bfloat16 stg[4][32][40];  // per epilogue warp: output staging
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int E = p.num_experts;
  const int feat_tiles = p.n / BN;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl.full[s], 1);   // used in the leader only
      mbar_init(&ctl.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl.acc_full[a], 1);
      mbar_init(&ctl.acc_empty[a], 2 * 4);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_act);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) tmem_alloc_2sm(&ctl.tmem_base, TMEM_COLS);
  if (warp == 2) build_tile_table(ctl, p.expert_offsets, p.dense_rows, E, BM2, feat_tiles, p.row_split);
  tcgen05_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tcgen05_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total_tiles = ctl.tile_start[E];

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs, one thread)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(&ctl.full[0]), 0);  // the leader's stage barriers
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_phase_mask = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
        const TileCoord tc = decode_tile(ctl, E, tile, BM2, feat_tiles);
        const int row0 = ctl.seg[tc.e] + tc.rblk * BM2;
        const int arow = (p.shared_a ? tc.rblk * BM2 : row0) + static_cast<int>(rank) * BM;
        const int wrow =
            (p.weight_mod ? tc.e % p.weight_mod : tc.e) * p.n + tc.fblk * BN + static_cast<int>(rank) * (BN / 2);
        int ka = 0;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          // the stage is free in this CTA once the leader's MMAs that read it completed
          if (!mbar_wait_cluster(&ctl.empty[stage], phase ^ 1u, &ctl.abort_flag, p.status)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&ctl.full[stage], 2 * STAGE_BYTES);
          const uint32_t bar = full0 + stage * static_cast<uint32_t>(sizeof(uint64_t));
          tma_load_2d_pair(sa + stage * A_BYTES, &tmap_act, bar, ka, arow);
          tma_load_2d_pair(sb + stage * B_BYTES, &tmap_w, bar, kb * BK, wrow);
          ka += BK;
          if (ka == p.k_blocks_a * BK) ka = 0;
          issued_mask |= 1u << stage;
          last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // let copies in flight land before the CTA exits: the leader watches
        // its stage barriers; the odd CTA cannot, and waits a fixed bounded time
        if (rank == 0) {
          for (int s = 0; s < STAGES; ++s)
            if ((issued_mask >> s) & 1u) drain_wait(&ctl.full[s], (last_phase_mask >> s) & 1u);
        } else if (issued_mask) {
          const long long t0 = clock64();
          while (clock64() - t0 < kWaitBudgetCycles / 64) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader CTA, one thread)
    if (rank == 0 && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(BM2, BN);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      int t_local = 0;
      for (int tile = pair; ok && tile < total_tiles; tile += npairs, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t acc_phase = (t_local >> 1) & 1;
        if (!mbar_wait_cluster(&ctl.acc_empty[acc], acc_phase ^ 1u, &ctl.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_cluster(&ctl.full[stage], phase, &ctl.abort_flag, p.status)) {
            ok = false;
            break;
          }
          const uint64_t da = umma_desc_sw128(smem_u32(sa + stage * A_BYTES));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / UK; ++k)
            umma_bf16_2sm(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_2sm(&ctl.empty[stage], 0x3);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_2sm(&ctl.acc_full[acc], 0x3);
      }
      if (!ok && issued) {
        umma_commit_2sm(&ctl.drain, 0x1);
        drain_wait(&ctl.drain, 0);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quarter = warp & 3;
    const int row_in_tile = static_cast<int>(rank) * BM + quarter * 32 + lane;
    const uint32_t acc_empty0 = mapa_shared(smem_u32(&ctl.acc_empty[0]), 0);
    int t_local = 0;
    for (int tile = pair; tile < total_tiles; tile += npairs, ++t_local) {
      const TileCoord tc = decode_tile(ctl, E, tile, BM2, feat_tiles);
      const int acc = t_local & 1;
      const uint32_t acc_phase = (t_local >> 1) & 1;
      const int seg_end = ctl.seg_end[tc.e];
      const int r = ctl.seg[tc.e] + tc.rblk * BM2 + row_in_tile;
      const bool valid = r < seg_end;
      const long long orow = valid ? (p.out_row_map ? p.out_row_map[r] : r) : 0;
      float scale = 1.f;
      if (p.epilogue == kEpiScaleBf16 && valid) scale = p.row_weight ? p.row_weight[r] : p.slot_weight[p.row_slot[r]];
      bool w = true;
      if (lane == 0) w = mbar_wait_cluster(&ctl.acc_full[acc], acc_phase, &ctl.abort_flag, p.status);
      if (!__shfl_sync(0xffffffffu, w ? 1 : 0, 0)) break;
      tcgen05_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      rows_epilogue<BN>(p, tbase, tc.fblk, orow, valid, scale, stg[quarter], lane);
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&ctl.acc_empty[acc]);
        else mbar_arrive_remote(acc_empty0 + acc * static_cast<uint32_t>(sizeof(uint64_t)));
      }
    }
  }

  tcgen05_fence_before();
  cluster_sync();  // both CTAs done with tensor memory and with each other's barriers
  tcgen05_fence_after();
  if (warp == 1) tmem_dealloc_2sm(tmem_base, TMEM_COLS);
}

// ============================================================ tokens schedule, SM pair
// Swap-AB tile on a 2-CTA cluster (tcgen05.mma.cta_group::2): 256 packed
// features are the MMA's M (weight rows, 128 per CTA) and up to 256 rows of
// one expert's segment are its N (half of the tile's rows loaded by each CTA).
// N is chosen per tile as the rows present rounded up to 16, so an expert's
// last, partial row block costs only the MMA work of the rows it holds (a
// 256-row M tile would pad it to 256).  Both CTAs' loads complete on the
// leader's stage barrier; the leader issues the MMAs; each CTA's TMEM holds
// D[its 128 features][N rows].  Epilogue: thread = feature, one 32-row chunk
// of the accumulator at a time; for SwiGLU the gate warp (features f) and the
// up warp (features f + 64) of the same 32 h columns swap half of each chunk
// through shared memory, so both compute 16 rows; a warp's 32 lanes store 32
// consecutive features (64 contiguous bytes) of one output row.
template <int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_tokens2_kernel(const __grid_constant__ CUtensorMap tmap_act,
                                const __grid_constant__ CUtensorMap tmap_w, const GroupedGemmParams p) {
  constexpr int BF = 2 * BM;                         // packed features per pair tile (MMA M)
  constexpr int BT = 256;                            // rows per tile at most (MMA N)
  constexpr uint32_t A_BYTES = BM * BK * 2;          // this CTA's 128 weight rows
  constexpr uint32_t B_BYTES = (BT / 2) * BK * 2;    // box of 128 activation rows (N/2 used)
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BT;
  static_assert(STAGES <= 16, "stages");

  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedCtl ctl;
  __shared__ float xch[2][2][2][32][17];  // [buffer][warp pair][0 gate, 1 up][lane][16 rows + pad]
  __shared__ __align__(16) __nv_bfloat16 stg[4][32][40];  // per epilogue warp: [row][32 features + pad]
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  const int E = p.num_experts;
  const int feat_tiles = p.n / BF;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl.full[s], 1);  // used in the leader only
      mbar_init(&ctl.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl.acc_full[a], 1);
      mbar_init(&ctl.acc_empty[a], 2 * 4);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_act);
    prefetch_tmap(&tmap_w);
  }
  if (warp == 1) tmem_alloc_2sm(&ctl.tmem_base, TMEM_COLS);
  if (warp == 2) build_tile_table(ctl, p.expert_offsets, p.dense_rows, E, BT, feat_tiles);
  tcgen05_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tcgen05_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total_tiles = ctl.tile_start[E];

  if (warp == 0) {
    // ---------------------------------------------------------------- producer (both CTAs, one thread)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(&ctl.full[0]), 0);  // the leader's stage barriers
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_phase_mask = 0;
      bool ok = true;
      for (int tile = pair; ok && tile < total_tiles; tile += npairs) {
        const TileCoord tc = decode_tile(ctl, E, tile, BT, feat_tiles);
        const int row0 = ctl.seg[tc.e] + tc.rblk * BT;
        const int nt = min(BT, ctl.seg_end[tc.e] - row0);
        const int half = ((nt + 15) & ~15) >> 1;  // rows of the MMA's N supplied by each CTA
        const int brow = (p.shared_a ? tc.rblk * BT : row0) + static_cast<int>(rank) * half;
        const int wrow = (p.weight_mod ? tc.e % p.weight_mod : tc.e) * p.n + tc.fblk * BF + static_cast<int>(rank) * BM;
        int ka = 0;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_cluster(&ctl.empty[stage], phase ^ 1u, &ctl.abort_flag, p.status)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&ctl.full[stage], 2 * STAGE_BYTES);
          const uint32_t bar = full0 + stage * static_cast<uint32_t>(sizeof(uint64_t));
          tma_load_2d_pair(sa + stage * A_BYTES, &tmap_w, bar, kb * BK, wrow);
          tma_load_2d_pair(sb + stage * B_BYTES, &tmap_act, bar, ka, brow);
          ka += BK;
          if (ka == p.k_blocks_a * BK) ka = 0;
          issued_mask |= 1u << stage;
          last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        if (rank == 0) {
          for (int s = 0; s < STAGES; ++s)
            if ((issued_mask >> s) & 1u) drain_wait(&ctl.full[s], (last_phase_mask >> s) & 1u);
        } else if (issued_mask) {
          const long long t0 = clock64();
          while (clock64() - t0 < kWaitBudgetCycles / 64) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader CTA, one thread)
    if (rank == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      int t_local = 0;
      for (int tile = pair; ok && tile < total_tiles; tile += npairs, ++t_local) {
        const TileCoord tc = decode_tile(ctl, E, tile, BT, feat_tiles);
        const int nt = min(BT, ctl.seg_end[tc.e] - ctl.seg[tc.e] - tc.rblk * BT);
        const uint32_t idesc = umma_idesc_bf16_f32(BF, (nt + 15) & ~15);
        const int acc = t_local & 1;
        const uint32_t acc_phase = (t_local >> 1) & 1;
        if (!mbar_wait_cluster(&ctl.acc_empty[acc], acc_phase ^ 1u, &ctl.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BT;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_cluster(&ctl.full[stage], phase, &ctl.abort_flag, p.status)) {
            ok = false;
            break;
          }
          const uint64_t da = umma_desc_sw128(smem_u32(sa + stage * A_BYTES));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / UK; ++k)
            umma_bf16_2sm(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma_commit_2sm(&ctl.empty[stage], 0x3);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_2sm(&ctl.acc_full[acc], 0x3);
      }
      if (!ok && issued) {
        umma_commit_2sm(&ctl.drain, 0x1);
        drain_wait(&ctl.drain, 0);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (both CTAs)
    const int quarter = warp & 3;       // TMEM lanes [32 quarter, 32 quarter + 32) = features
    const int wpair = quarter & 1;      // SwiGLU: gate quarter q pairs with up quarter q + 2
    const bool is_up = quarter >= 2;
    const uint32_t acc_empty0 = mapa_shared(smem_u32(&ctl.acc_empty[0]), 0);
    int t_local = 0;
    for (int tile = pair; tile < total_tiles; tile += npairs, ++t_local) {
      const TileCoord tc = decode_tile(ctl, E, tile, BT, feat_tiles);
      const int acc = t_local & 1;
      const uint32_t acc_phase = (t_local >> 1) & 1;
      const int row0 = ctl.seg[tc.e] + tc.rblk * BT;
      const int nt = min(BT, ctl.seg_end[tc.e] - row0);
      bool ok = true;
      if (lane == 0) ok = mbar_wait_cluster(&ctl.acc_full[acc], acc_phase, &ctl.abort_flag, p.status);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      // the SwiGLU hand-off uses named barriers between warps: all four take
      // the same path, so stopping is a vote over the 128 epilogue threads
      if (named_bar_any(1, 128, !ok)) break;
      tcgen05_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BT;
      // Output rows leave through the warp's staging tile: thread = feature
      // writes its column, then lane l stores 16 bytes (8 features) of row
      // l / 4 + 8 i, so a store instruction covers 8 rows x 64 bytes.
      __nv_bfloat16(*st)[40] = stg[quarter];
      __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
      if (p.epilogue == kEpiSwiGLU) {
        const long long hcol0 = static_cast<long long>(tc.fblk) * (BF / 2) + rank * (BM / 2) + wpair * 32;
        int buf = 0;
        for (int c = 0; c < nt; c += 32, buf ^= 1) {
          float v[32];
          tmem_ld_cols<32>(taddr + c, v);
          // the gate warp computes rows c..c+15, the up warp rows c+16..c+31
#pragma unroll
          for (int j = 0; j < 16; ++j) xch[buf][wpair][is_up ? 1 : 0][lane][j] = is_up ? v[j] : v[16 + j];
          named_bar_sync(2 + wpair, 64);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float g = is_up ? xch[buf][wpair][0][lane][j] : v[j];
            const float u = is_up ? v[16 + j] : xch[buf][wpair][1][lane][j];
            st[j][lane] = __float2bfloat16_rn(silu_f(g) * u);
          }
          __syncwarp();
          const int c0 = c + (is_up ? 16 : 0);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int rr = (lane >> 2) + 8 * i;
            if (c0 + rr < nt) {
              const long long r = row0 + c0 + rr;
              const long long orow = p.out_row_map ? p.out_row_map[r] : r;
              *reinterpret_cast<uint4*>(out + orow * p.out_ld + hcol0 + (lane & 3) * 8) =
                  *reinterpret_cast<const uint4*>(&st[rr][(lane & 3) * 8]);
            }
          }
          __syncwarp();
        }
      } else {  // kEpiScaleBf16 / kEpiStoreBf16
        const long long col0 = static_cast<long long>(tc.fblk) * BF + rank * BM + quarter * 32;
        for (int c = 0; c < nt; c += 32) {
          float v[32];
          tmem_ld_cols<32>(taddr + c, v);
          if (p.epilogue == kEpiScaleBf16) {
            const int rl = row0 + c + lane;
            const float wl =
                (c + lane < nt) ? (p.row_weight ? p.row_weight[rl] : p.slot_weight[p.row_slot[rl]]) : 0.f;
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] *= __shfl_sync(0xffffffffu, wl, j);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) st[j][lane] = __float2bfloat16_rn(v[j]);
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int rr = (lane >> 2) + 8 * i;
            if (c + rr < nt) {
              const long long r = row0 + c + rr;
              const long long orow = p.out_row_map ? p.out_row_map[r] : r;
              *reinterpret_cast<uint4*>(out + orow * p.out_ld + col0 + (lane & 3) * 8) =
                  *reinterpret_cast<const uint4*>(&st[rr][(lane & 3) * 8]);
            }
          }
          __syncwarp();
        }
      }
      tcgen05_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0) mbar_arrive(&ctl.acc_empty[acc]);
        else mbar_arrive_remote(acc_empty0 + acc * static_cast<uint32_t>(sizeof(uint64_t)));
      }
    }
  }

  tcgen05_fence_before();
  cluster_sync();  // both CTAs done with tensor memory and with each other's barriers
  tcgen05_fence_after();
  if (warp == 1) tmem_dealloc_2sm(tmem_base, TMEM_COLS);
}

// ============================================================ weights schedule
// Tile: 128 packed features x BT activation rows.  A = weight block (box 64 x
// 128), B = activation rows (box 64 x BT); D[feature][row].
template <int BT, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_weights_kernel(const __grid_constant__ CUtensorMap tmap_act,
                                const __grid_constant__ CUtensorMap tmap_w, const GroupedGemmParams p) {
  constexpr uint32_t A_BYTES = BM * BK * 2;  // weight block
  constexpr uint32_t B_BYTES = BT * BK * 2;  // activation rows
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = (2 * BT < 32) ? 32 : 2 * BT;
  static_assert(STAGES <= 16, "stages");

  extern __shared__ uint8_t smem_raw[];
  __shared__ SharedCtl ctl;
  __shared__ float xch[64][BT + 1];  // up-projection values handed to the gate lanes
  uint8_t* smem = align1024(smem_raw);
  uint8_t* sa = smem;
  uint8_t* sb = smem + STAGES * A_BYTES;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = p.num_experts;
  const int feat_tiles = p.n / BM;

  const bool gather_a = p.a_row_map != nullptr;
  const bool gather_cp = gather_a && !p.tma_gather4;  // rows written by cp.async (generic proxy)
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&ctl.full[s], gather_cp ? 1 + 32 : 1);  // + one cp.async arrival per producer lane
      mbar_init(&ctl.empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&ctl.acc_full[a], 1);
      mbar_init(&ctl.acc_empty[a], 4 * 32);
    }
    mbar_init(&ctl.drain, 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_act);
    prefetch_tmap(&tmap_w);
  }
  // programmatic dependent launch: the prologue above overlaps the previous
  // kernel; its outputs (offsets, activation rows) are read after this wait
  pdl_launch_dependents();
  pdl_wait();
  if (warp == 1) tmem_alloc(&ctl.tmem_base, TMEM_COLS);
  if (warp == 2) build_tile_table(ctl, p.expert_offsets, p.dense_rows, E, BT, feat_tiles);
  tcgen05_fence_before();
  __syncthreads();
  tcgen05_fence_after();
  const uint32_t tmem_base = ctl.tmem_base;
  const int total_tiles = ctl.tile_start[E];
  // balance_waves: the tiles dealt to as many CTAs as their waves need
  // (ceil(tiles / ceil(tiles / grid))), so the weight stream does not end with
  // a few CTAs reading alone; the other CTAs take no tile
  int ncta = static_cast<int>(gridDim.x);
  if (p.balance_waves && total_tiles > 0) {
    const int waves = (total_tiles + ncta - 1) / ncta;
    ncta = (total_tiles + waves - 1) / waves;
  }
  const int first_tile = static_cast<int>(blockIdx.x) < ncta ? static_cast<int>(blockIdx.x) : total_tiles;

  if (warp == 0) {
    // TMA mode: lane 0 alone runs the loop; gather mode: the whole warp
    if (gather_a || lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, last_phase_mask = 0;
      bool ok = true;
      const uint64_t pol_w = policy_evict_first();
      for (int tile = first_tile; ok && tile < total_tiles; tile += ncta) {
        const TileCoord tc = decode_tile(ctl, E, tile, BT, feat_tiles);
        const int row0 = ctl.seg[tc.e] + tc.rblk * BT;
        const int arow0 = p.shared_a ? tc.rblk * BT : row0;
        const int wrow0 = (p.weight_mod ? tc.e % p.weight_mod : tc.e) * p.n + tc.fblk * BM;
        // cp.async gather: tile row lane + 32 j; TMA gather4: lanes < BT / 4
        // load tile rows 4 lane + j (rows past the segment end re-read the
        // tile's first row; their accumulator columns are never stored)
        int src_row[(BT + 31) / 32];
        int g4[4];
        if (gather_cp) {
          const int seg_end = ctl.seg_end[tc.e];
#pragma unroll
          for (int j = 0; j < (BT + 31) / 32; ++j) {
            const int r = row0 + lane + 32 * j;
            src_row[j] = (lane + 32 * j < BT && r < seg_end) ? p.a_row_map[r] : -1;
          }
        } else if (gather_a) {
          const int seg_end = ctl.seg_end[tc.e];
          const int first = p.a_row_map[row0];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int r = row0 + 4 * lane + j;
            g4[j] = (4 * lane + j < BT && r < seg_end) ? p.a_row_map[r] : first;
          }
        }
        int ka = 0;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (gather_a) {
            if (!warp_wait(&ctl.empty[stage], phase ^ 1u, ctl, p.status)) {
              ok = false;
              break;
            }
            if (lane == 0) {
              mbar_arrive_expect_tx(&ctl.full[stage], gather_cp ? A_BYTES : STAGE_BYTES);
              tma_load_2d_hint(sa + stage * A_BYTES, &tmap_w, &ctl.full[stage], kb * BK, wrow0, pol_w);
            }
            if (gather_cp) {
              gather_k_block<BT>(smem_u32(sb + stage * B_BYTES), p.a_ptr, p.a_ld, ka, src_row, lane);
              cp_async_mbar_arrive(&ctl.full[stage]);
            } else {  // BT / 4 lanes x 4 rows x 128 bytes = the BT-row B stage
              __syncwarp();
              if (lane < BT / 4)
                tma_gather4_2d(sb + stage * B_BYTES + lane * 512, &tmap_act, &ctl.full[stage], ka, g4[0], g4[1],
                               g4[2], g4[3]);
            }
          } else {
            if (!mbar_wait(&ctl.empty[stage], phase ^ 1u, &ctl.abort_flag, p.status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&ctl.full[stage], STAGE_BYTES);
            tma_load_2d_hint(sa + stage * A_BYTES, &tmap_w, &ctl.full[stage], kb * BK, wrow0, pol_w);
            tma_load_2d(sb + stage * B_BYTES, &tmap_act, &ctl.full[stage], ka, arow0);
          }
          ka += BK;
          if (ka == p.k_blocks_a * BK) ka = 0;
          issued_mask |= 1u << stage;
          last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && lane == 0) {
        for (int s = 0; s < STAGES; ++s)
          if ((issued_mask >> s) & 1u) drain_wait(&ctl.full[s], (last_phase_mask >> s) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {  // one thread issues every MMA and commit
      constexpr uint32_t idesc = umma_idesc_bf16_f32(BM, BT);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true, issued = false;
      int t_local = 0;
      for (int tile = first_tile; ok && tile < total_tiles; tile += ncta, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t acc_phase = (t_local >> 1) & 1;
        if (!mbar_wait(&ctl.acc_empty[acc], acc_phase ^ 1u, &ctl.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tcgen05_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BT;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&ctl.full[stage], phase, &ctl.abort_flag, p.status)) {
            ok = false;
            break;
          }
          if (gather_cp) fence_proxy_async_shared();  // cp.async-written B -> tensor-core reads
          const uint64_t da = umma_desc_sw128(smem_u32(sa + stage * A_BYTES));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + stage * B_BYTES));
#pragma unroll
          for (int kq = 0; kq < BK / UK; ++kq)
            umma_bf16(d_tmem, da + 2 * kq, db + 2 * kq, idesc, (kb | kq) != 0 ? 1u : 0u);
          umma_commit(&ctl.empty[stage]);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&ctl.acc_full[acc]);
      }
      if (!ok && issued) {
        umma_commit(&ctl.drain);
        drain_wait(&ctl.drain, 0);
      }
    }
    __syncwarp();
  } else {
    const int quarter = warp & 3;
    const int feat = quarter * 32 + lane;  // TMEM lane = feature row of the tile
    int t_local = 0;
    for (int tile = first_tile; tile < total_tiles; tile += ncta, ++t_local) {
      const TileCoord tc = decode_tile(ctl, E, tile, BT, feat_tiles);
      const int acc = t_local & 1;
      const uint32_t acc_phase = (t_local >> 1) & 1;
      const bool ok = warp_wait(&ctl.acc_full[acc], acc_phase, ctl, p.status);
      // the SwiGLU hand-off below uses a named barrier over all four warps:
      // every epilogue warp must take the same path, so the stop decision is
      // a vote over all 128 threads
      if (named_bar_any(1, 128, !ok)) break;
      tcgen05_fence_after();
      const int r0 = ctl.seg[tc.e] + tc.rblk * BT;
      const int nvalid = min(BT, ctl.seg_end[tc.e] - r0);
      float v[BT];
      tmem_ld_cols<BT>(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BT, v);
      tcgen05_fence_before();
      mbar_arrive(&ctl.acc_empty[acc]);  // accumulator is in registers now

      if (p.epilogue == kEpiSwiGLU) {
        // lanes 0-63: gate of feature tc.fblk*64 + feat; lanes 64-127: up of feature - 64
        if (feat >= 64) {
#pragma unroll
          for (int j = 0; j < BT; ++j) xch[feat - 64][j] = v[j];
        }
        named_bar_sync(1, 128);
        if (feat < 64) {
          __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
          const long long col = static_cast<long long>(tc.fblk) * 64 + feat;
#pragma unroll
          for (int j = 0; j < BT; ++j) {
            if (j >= nvalid) break;
            const long long r = r0 + j;
            const long long orow = p.out_row_map ? p.out_row_map[r] : r;
            out[orow * p.out_ld + col] = __float2bfloat16_rn(silu_f(v[j]) * xch[feat][j]);
          }
        }
      } else if (p.epilogue == kEpiScaleBf16 || p.epilogue == kEpiStoreBf16) {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
        const long long col = static_cast<long long>(tc.fblk) * BM + feat;
#pragma unroll
        for (int j = 0; j < BT; ++j) {
          if (j >= nvalid) break;
          const long long r = r0 + j;
          const float sc = p.epilogue != kEpiScaleBf16 ? 1.f : (p.row_weight ? p.row_weight[r] : p.slot_weight[p.row_slot[r]]);
          const long long orow = p.out_row_map ? p.out_row_map[r] : r;
          out[orow * p.out_ld + col] = __float2bfloat16_rn(sc * v[j]);
        }
      } else {
        float* out = static_cast<float*>(p.out);
        const long long col = static_cast<long long>(tc.fblk) * BM + feat;
        const float b = p.col_bias ? p.col_bias[col] : 0.f;
#pragma unroll
        for (int j = 0; j < BT; ++j) {
          if (j >= nvalid) break;
          const long long r = r0 + j;
          const long long orow = p.out_row_map ? p.out_row_map[r] : r;
          out[orow * p.out_ld + col] = v[j] + b;
        }
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tcgen05_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// The dynamic shared-memory opt-in is set once per kernel and device (not
// per launch), so launches can be captured into CUDA graphs.
using GemmKernel = void (*)(CUtensorMap, CUtensorMap, GroupedGemmParams);

cudaError_t ensure_smem_optin(GemmKernel kernel, size_t smem) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;  // (kernel, device)
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) done.insert(key);
  return e;
}

cudaError_t launch_with_smem(GemmKernel kernel, size_t smem, int grid, const CUtensorMap& a, const CUtensorMap& w,
                             const GroupedGemmParams& p, cudaStream_t s, bool pdl = false) {
  cudaError_t e = ensure_smem_optin(kernel, smem);
  if (e != cudaSuccess) return e;
  if (pdl) return launch_pdl(kernel, dim3(grid), dim3(kThreads), smem, s, a, w, p);
  kernel<<<grid, kThreads, smem, s>>>(a, w, p);
  return cudaGetLastError();
}

// Co-resident 2-CTA clusters of `kernel` on the current device (a TPC with a
// disabled SM cannot host one), cached per (kernel, device).  A persistent
// grid larger than this would run its last clusters after the others finish.
int max_active_pairs(GemmKernel kernel, const cudaLaunchConfig_t& cfg_in) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = cfg_in;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = device_sm_count() / 2;
  }
  cache[key] = n;
  return n;
}

cudaError_t launch_cluster2(GemmKernel kernel, size_t smem, int grid, const CUtensorMap& a, const CUtensorMap& w,
                            const GroupedGemmParams& p, cudaStream_t s) {
  cudaError_t e = ensure_smem_optin(kernel, smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(2, 1, 1);
  const int pairs = std::max(1, std::min(grid / 2, max_active_pairs(kernel, cfg)));
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kernel, a, w, p);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

constexpr size_t rows2_smem(int bn, int stages) {
  return static_cast<size_t>(stages) * (BM * BK * 2 + (bn / 2) * BK * 2) + 1024;
}

constexpr size_t tokens2_smem(int stages) { return static_cast<size_t>(stages) * (BM * BK * 2 + 128 * BK * 2) + 1024; }

constexpr size_t rows_smem(int bn, int stages) { return static_cast<size_t>(stages) * (BM * BK * 2 + bn * BK * 2) + 1024; }
constexpr size_t weights_smem(int bt, int stages) {
  return static_cast<size_t>(stages) * (BM * BK * 2 + bt * BK * 2) + 1024;
}

}  // namespace

int grouped_gemm_box_rows_act(int variant) {
  switch (variant) {
    case kRowsBN256:
    case kRowsBN128:
    case kRows2BN256: return BM;
    case kTokens2: return 128;  // up to 128 of the tile's rows per CTA
    case kWeightsT16: return 16;
    case kWeightsT32: return 32;
    case kWeightsT64: return 64;
  }
  return 0;
}

int grouped_gemm_box_rows_w(int variant) {
  switch (variant) {
    case kRowsBN256: return 256;
    case kRowsBN128: return 128;
    case kRows2BN256: return 128;  // each CTA of the pair loads half of the 256 features
    default: return BM;
  }
}

cudaError_t grouped_gemm_launch(int variant, const CUtensorMap& tmap_act, const CUtensorMap& tmap_w,
                                const GroupedGemmParams& p, int grid, cudaStream_t s) {
  switch (variant) {
    case kRowsBN256:
      return launch_with_smem(grouped_gemm_rows_kernel<256, 4>, rows_smem(256, 4), grid, tmap_act, tmap_w, p, s);
    case kRowsBN128:
      return launch_with_smem(grouped_gemm_rows_kernel<128, 6>, rows_smem(128, 6), grid, tmap_act, tmap_w, p, s);
    case kRows2BN256:
      if (grid % 2) return cudaErrorInvalidValue;
      return launch_cluster2(grouped_gemm_rows2_kernel<256, 6>, rows2_smem(256, 6), grid, tmap_act, tmap_w, p, s);
    case kTokens2:
      if (grid % 2 || (p.epilogue != kEpiSwiGLU && p.epilogue != kEpiScaleBf16 && p.epilogue != kEpiStoreBf16) ||
          p.n % 256 != 0 || p.a_row_map)
        return cudaErrorInvalidValue;
      return launch_cluster2(grouped_gemm_tokens2_kernel<6>, tokens2_smem(6), grid, tmap_act, tmap_w, p, s);
    case kWeightsT16:
      return launch_with_smem(grouped_gemm_weights_kernel<16, 8>, weights_smem(16, 8), grid, tmap_act, tmap_w, p, s,
                              true);
    case kWeightsT32:
      return launch_with_smem(grouped_gemm_weights_kernel<32, 8>, weights_smem(32, 8), grid, tmap_act, tmap_w, p, s,
                              true);
    case kWeightsT64:
      return launch_with_smem(grouped_gemm_weights_kernel<64, 6>, weights_smem(64, 6), grid, tmap_act, tmap_w, p, s,
                              true);
  }
  return cudaErrorInvalidValue;
}

}  // namespace nkimoe
