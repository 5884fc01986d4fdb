// Skinny linear layer for decode: y[M, N] = x[M, K] . w[N, K]^T with M <= 16
// (bf16 in and out, fp32 accumulation).  At M <= 16 the product is bound by
// reading w once from HBM; the kernel streams it at that rate.
//
// Reference: the projections of the decode step (nki_qkv_projection,
// nki_attention.py:32-169, and the O projection of the attention block,
// qwen_with_nki.py:330-350); the NKI generic tile matmul is nki_matmul_tiled
// (nki_moe_integrated.py:27-84).
//
// CTA = 16 rows of w (the MMA's M, "swap AB": the weight rows are the A
// operand, the tokens the N = 8 columns), the whole K range split over 8
// warps.  A lane (g = lane / 4, t = lane % 4) loads 16 bytes of w rows g and
// g + 8 and of token row g at k = k0 + 8t .. 8t + 7 for every 32-wide block
// k0.  The MMA contracts over 16 k per instruction in a fixed lane layout; the
// dot product does not depend on the order of k, so the same permutation of k
// is applied to both operands and the loaded vectors are the fragments as
// they are: elements 0-3 of each vector feed one m16n8k16 MMA and elements
// 4-7 the next.  The 8 warps' partial tiles are added in warp order through
// shared memory (deterministic).
#include "kernels.h"

namespace nkimoe {

namespace {

constexpr int kLinWarps = 8;
constexpr int kLinUnroll = 8;  // 32-wide k blocks per warp with loads in flight together

__device__ __forceinline__ void mma_16816_lin(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_stream(const __nv_bfloat16* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// MT: token tiles of 8 (M <= 8 * MT)
template <int MT>
__global__ void __launch_bounds__(kLinWarps * 32) skinny_linear_kernel(const __nv_bfloat16* __restrict__ x,
                                                                      const __nv_bfloat16* __restrict__ w,
                                                                      __nv_bfloat16* __restrict__ y, int M, int N,
                                                                      int K) {
  __shared__ float red[kLinWarps][MT][16][9];  // padded: conflict-free column reads
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const long long n0 = static_cast<long long>(blockIdx.x) * 16;
  const __nv_bfloat16* w0 = w + (n0 + g) * K + 8 * t;
  const __nv_bfloat16* w1 = w0 + 8LL * K;
  const __nv_bfloat16* xr[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int m = mt * 8 + g;
    xr[mt] = x + static_cast<long long>(m < M ? m : 0) * K + 8 * t;  // rows past M: any valid row, not stored
  }
  float acc[MT][4] = {};
  const int blocks = K >> 5;
  for (int b0 = warp; b0 < blocks; b0 += kLinWarps * kLinUnroll) {
    uint4 wa[kLinUnroll], wb[kLinUnroll], xv[kLinUnroll][MT];
#pragma unroll
    for (int u = 0; u < kLinUnroll; ++u) {
      const int b = b0 + u * kLinWarps;
      if (b < blocks) {
        wa[u] = ldg_stream(w0 + 32LL * b);
        wb[u] = ldg_stream(w1 + 32LL * b);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) xv[u][mt] = *reinterpret_cast<const uint4*>(xr[mt] + 32LL * b);
      }
    }
#pragma unroll
    for (int u = 0; u < kLinUnroll; ++u) {
      if (b0 + u * kLinWarps < blocks) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma_16816_lin(acc[mt], wa[u].x, wb[u].x, wa[u].y, wb[u].y, xv[u][mt].x, xv[u][mt].y);
          mma_16816_lin(acc[mt], wa[u].z, wb[u].z, wa[u].w, wb[u].w, xv[u][mt].z, xv[u][mt].w);
        }
      }
    }
  }
  // acc[mt]: rows g / g + 8 of the CTA's 16 weight rows, tokens mt*8 + 2t, +1
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    red[warp][mt][g][2 * t] = acc[mt][0];
    red[warp][mt][g][2 * t + 1] = acc[mt][1];
    red[warp][mt][g + 8][2 * t] = acc[mt][2];
    red[warp][mt][g + 8][2 * t + 1] = acc[mt][3];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < MT * 128; o += kLinWarps * 32) {
    const int mt = o >> 7, c = (o >> 4) & 7, r = o & 15;  // 16 threads: 16 consecutive outputs of a token
    const int m = mt * 8 + c;
    float s = red[0][mt][r][c];
#pragma unroll
    for (int ww = 1; ww < kLinWarps; ++ww) s += red[ww][mt][r][c];
    if (m < M) y[static_cast<long long>(m) * N + n0 + r] = __float2bfloat16_rn(s);
  }
}

}  // namespace

cudaError_t skinny_linear_launch(const __nv_bfloat16* x, const __nv_bfloat16* w, __nv_bfloat16* y, int M, int N,
                                 int K, cudaStream_t s) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (M < 0 || M > 16 || N % 16 != 0 || K % 32 != 0 || K <= 0) return cudaErrorInvalidValue;
  // one CTA per 16 weight rows (a K split over CTA clusters, partials added
  // through distributed shared memory, measured slower at every shape here)
  const unsigned grid = static_cast<unsigned>(N / 16);
  cudaError_t e = M <= 8 ? launch_pdl(skinny_linear_kernel<1>, dim3(grid), dim3(kLinWarps * 32), 0, s, x, w, y, M, N, K)
                         : launch_pdl(skinny_linear_kernel<2>, dim3(grid), dim3(kLinWarps * 32), 0, s, x, w, y, M, N, K);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace nkimoe
