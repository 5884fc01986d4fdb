// One-time expert-weight re-layout for the tcgen05 GEMMs.
//
// The reference keeps gate_up_proj as [E, H, 2I] (gate columns 0..I-1, up
// columns I..2I-1) and down_proj as [E, I, H] (qwen.py:164-226).  The GEMMs
// want both operands K-major (the reduction dimension contiguous), so:
//   W13[e] : [2I, H], row blocks of 128 = [gate rows 64b..64b+63 | up rows 64b..64b+63]
//   W2[e]  : [H, I]  (plain transpose of down_proj[e])
// The 64-row gate/up interleave puts the gate and up accumulators of the same
// features in one 128-feature tile, so the SwiGLU is applied in the GEMM
// epilogue without a second pass.  HF transformers stores gate_up_proj as
// [E, 2I, H] already; for it the packing is a row permutation.
#include "kernels.h"

namespace nkimoe {

namespace {

__device__ __forceinline__ int packed_row(int c, int inter) {
  const int up = c >= inter;
  const int j = up ? c - inter : c;
  return (j >> 6) * 128 + up * 64 + (j & 63);
}

// in [B][R][C] -> out [B][C'][R], C' = packed_row(c) when inter > 0 else c.
__global__ void transpose_pack_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int R,
                                      int C, int inter) {
  __shared__ __nv_bfloat16 tile[32][33];
  const long long b = blockIdx.z;
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const __nv_bfloat16* src = in + b * R * C;
  __nv_bfloat16* dst = out + b * R * C;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int r = r0 + threadIdx.y + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[threadIdx.y + i][threadIdx.x] = src[static_cast<long long>(r) * C + c];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int c = c0 + threadIdx.y + i, r = r0 + threadIdx.x;
    if (r < R && c < C) {
      const int cp = inter > 0 ? packed_row(c, inter) : c;
      dst[static_cast<long long>(cp) * R + r] = tile[threadIdx.x][threadIdx.y + i];
    }
  }
}

// in [E][2I][H] -> out rows permuted into the packed order (16-byte moves).
__global__ void permute_rows_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out,
                                    long long rows_total, int rows_per_expert, int H, int inter) {
  const int chunks = H >> 3;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows_total * chunks;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i / chunks;
    const int ch = static_cast<int>(i % chunks);
    const long long e = row / rows_per_expert;
    const int c = static_cast<int>(row % rows_per_expert);
    const long long dst_row = e * rows_per_expert + packed_row(c, inter);
    reinterpret_cast<uint4*>(out + dst_row * H)[ch] = reinterpret_cast<const uint4*>(in + row * H)[ch];
  }
}

}  // namespace

cudaError_t pack_gate_up_nxd_launch(const __nv_bfloat16* in, __nv_bfloat16* out, int experts, int hidden, int inter,
                                    cudaStream_t s) {
  if (inter % 64 || hidden % 32) return cudaErrorInvalidValue;
  dim3 grid((2 * inter + 31) / 32, (hidden + 31) / 32, experts);
  transpose_pack_kernel<<<grid, dim3(32, 8), 0, s>>>(in, out, hidden, 2 * inter, inter);
  return cudaGetLastError();
}

cudaError_t pack_gate_up_hf_launch(const __nv_bfloat16* in, __nv_bfloat16* out, int experts, int hidden, int inter,
                                   cudaStream_t s) {
  if (inter % 64 || hidden % 8) return cudaErrorInvalidValue;
  const long long rows = static_cast<long long>(experts) * 2 * inter;
  const long long work = rows * (hidden / 8);
  const unsigned blocks = static_cast<unsigned>(std::min<long long>((work + 255) / 256, 1 << 20));
  permute_rows_kernel<<<blocks, 256, 0, s>>>(in, out, rows, 2 * inter, hidden, inter);
  return cudaGetLastError();
}

cudaError_t transpose_launch(const __nv_bfloat16* in, __nv_bfloat16* out, int batch, int rows, int cols,
                             cudaStream_t s) {
  dim3 grid((cols + 31) / 32, (rows + 31) / 32, batch);
  transpose_pack_kernel<<<grid, dim3(32, 8), 0, s>>>(in, out, rows, cols, 0);
  return cudaGetLastError();
}

}  // namespace nkimoe
