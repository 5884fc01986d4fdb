// K1: RMSNorm over rows of a [rows, hidden] tensor (nki_custom_rmsnorm.py:8-70)
//     y = x * rsqrt(mean(x^2) + eps) * w, fp32 arithmetic, one warp per row,
//     128-bit loads/stores.  Optional fused residual add in front of it
//     (the decoder's `h = h + attn; post_attention_layernorm(h)`,
//     qwen_with_nki.py:447-452).
// K6: per-head q/k RMSNorm + rotate-half RoPE on a fused [Q | K | V] row
//     (qwen_with_nki.py:330-350 with the HF Qwen3-MoE order: norm, then RoPE).
#include <type_traits>

#include "kernels.h"
#include "rope.cuh"

namespace nkimoe {

namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  float4 a = *reinterpret_cast<const float4*>(p);
  float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void round_bf16(float (&v)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = __bfloat162float(__float2bfloat16_rn(v[j]));
}

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16x2(v[0], v[1]);
  u.y = pack_bf16x2(v[2], v[3]);
  u.z = pack_bf16x2(v[4], v[5]);
  u.w = pack_bf16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}

__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Rows of up to kMaxChunks*8*32 elements are held in registers (one pass over
// HBM); longer rows are re-read from L2 for the second pass.
constexpr int kMaxChunks = 8;  // 2048 elements per row in registers

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

// bf16 rows: the register-held part of a row stays packed (4 registers per 8
// elements instead of 8), so more warps fit on an SM and more of the rows'
// loads are in flight; the arithmetic and its order are those of the generic
// kernel below.
template <typename TW, typename TO, bool kResidual>
__global__ void __launch_bounds__(256, 3) rmsnorm_bf16_kernel(const __nv_bfloat16* x, const __nv_bfloat16* residual,
                                                           __nv_bfloat16* residual_out, const TW* __restrict__ w,
                                                           TO* out, long long rows, int hidden, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nchunk = hidden >> 3;
  const __nv_bfloat16* xr = x + row * hidden;
  uint4 p[kMaxChunks];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) p[i] = *reinterpret_cast<const uint4*>(xr + c * 8);
  }
  if constexpr (kResidual) {
    uint4 q[kMaxChunks];
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + i * 32;
      if (c < nchunk) q[i] = *reinterpret_cast<const uint4*>(residual + row * hidden + c * 8);
    }
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + i * 32;
      if (c < nchunk) {
        float v[8], r[8];
        unpack8(p[i], v);
        unpack8(q[i], r);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += r[j];
        // the sum is rounded to the residual stream's dtype before the norm
        p[i].x = pack_bf16x2(v[0], v[1]);
        p[i].y = pack_bf16x2(v[2], v[3]);
        p[i].z = pack_bf16x2(v[4], v[5]);
        p[i].w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(residual_out + row * hidden + c * 8) = p[i];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) {
      float v[8];
      unpack8(p[i], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[j], v[j], ss);
    }
  }
  for (int c = lane + kMaxChunks * 32; c < nchunk; c += 32) {
    float t[8];
    if constexpr (kResidual) {
      float r[8];
      load8(xr + c * 8, t);
      load8(residual + row * hidden + c * 8, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] += r[j];
      round_bf16(t);
      store8(residual_out + row * hidden + c * 8, t);
    } else {
      load8(xr + c * 8, t);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(t[j], t[j], ss);
  }
  ss = warp_sum(ss);
  const float rinv = rsqrtf(ss / static_cast<float>(hidden) + eps);
  TO* orow = out + row * hidden;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) {
      float v[8], wv[8], o[8];
      unpack8(p[i], v);
      load8(w + c * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[j] * rinv * wv[j];
      store8(orow + c * 8, o);
    }
  }
  const __nv_bfloat16* src = kResidual ? residual_out + row * hidden : xr;
  for (int c = lane + kMaxChunks * 32; c < nchunk; c += 32) {
    float t[8], wv[8];
    load8(src + c * 8, t);
    load8(w + c * 8, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = t[j] * rinv * wv[j];
    store8(orow + c * 8, t);
  }
}

template <typename TX, typename TW, typename TO, bool kResidual>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const TX* x, const TX* residual, TX* residual_out,
                                                      const TW* __restrict__ w, TO* out, long long rows, int hidden, float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nchunk = hidden >> 3;  // 8-element chunks
  const TX* xr = x + row * hidden;
  float v[kMaxChunks][8];
  float ss = 0.f;
  // Every load of the register-held part of the row is issued before any
  // store: x, residual and residual_out may alias (in-place residual update),
  // so a store between them would serialise the loads one round trip each.
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) load8(xr + c * 8, v[i]);
  }
  if constexpr (kResidual) {
    float r[kMaxChunks][8];
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + i * 32;
      if (c < nchunk) load8(residual + row * hidden + c * 8, r[i]);
    }
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int c = lane + i * 32;
      if (c < nchunk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[i][j];
        // the sum is rounded to the residual stream's dtype before the norm
        round_bf16(v[i]);
        store8(residual_out + row * hidden + c * 8, v[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) {
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    }
  }
  for (int c = lane + kMaxChunks * 32; c < nchunk; c += 32) {
    float t[8];
    if constexpr (kResidual) {
      float r[8];
      load8(xr + c * 8, t);
      load8(residual + row * hidden + c * 8, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) t[j] += r[j];
      round_bf16(t);
      store8(residual_out + row * hidden + c * 8, t);
    } else {
      load8(xr + c * 8, t);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = fmaf(t[j], t[j], ss);
  }
  ss = warp_sum(ss);
  const float rinv = rsqrtf(ss / static_cast<float>(hidden) + eps);
  TO* orow = out + row * hidden;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int c = lane + i * 32;
    if (c < nchunk) {
      float wv[8], o[8];
      load8(w + c * 8, wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rinv * wv[j];
      store8(orow + c * 8, o);
    }
  }
  const TX* src = kResidual ? residual_out + row * hidden : xr;
  for (int c = lane + kMaxChunks * 32; c < nchunk; c += 32) {
    float t[8], wv[8];
    load8(src + c * 8, t);
    load8(w + c * 8, wv);
#pragma unroll
    for (int j = 0; j < 8; ++j) t[j] = t[j] * rinv * wv[j];
    store8(orow + c * 8, t);
  }
}

// Few rows (a decode step): one CTA per row so that the row's loads are spread
// over 256 threads and all of them -- x, residual and the norm weight -- are
// in flight at once; the sum of squares is reduced across the CTA.  Rows of
// up to kRowChunks * 8 * 256 elements.
constexpr int kRowThreads = 256;
constexpr int kRowChunks = 4;

template <typename TX, typename TW, typename TO, bool kResidual>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_row_kernel(const TX* x, const TX* residual, TX* residual_out,
                                                                  const TW* __restrict__ w, TO* out, int hidden,
                                                                  float eps) {
  __shared__ float red[kRowThreads / 32];
  pdl_launch_dependents();
  pdl_wait();
  const long long row = blockIdx.x;
  const int nchunk = hidden >> 3;
  float v[kRowChunks][8], wv[kRowChunks][8];
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
      load8(x + row * hidden + c * 8, v[i]);
      load8(w + c * 8, wv[i]);
    }
  }
  if constexpr (kResidual) {
    float r[kRowChunks][8];
#pragma unroll
    for (int i = 0; i < kRowChunks; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nchunk) load8(residual + row * hidden + c * 8, r[i]);
    }
#pragma unroll
    for (int i = 0; i < kRowChunks; ++i) {
      const int c = threadIdx.x + i * kRowThreads;
      if (c < nchunk) {
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] += r[i][j];
        round_bf16(v[i]);
        store8(residual_out + row * hidden + c * 8, v[i]);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRowThreads / 32; ++k) ss += red[k];
  const float rinv = rsqrtf(ss / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rinv * wv[i][j];
      store8(out + row * hidden + c * 8, o);
    }
  }
}

// The MoE block's combine fused with the decoder's next residual add +
// RMSNorm, for few rows: per token row (one CTA), h = sum_k y[slot_row[t,k]]
// in fp32 with k ascending and rounded to bf16 (combine_kernel's arithmetic),
// then r = h + residual rounded to bf16 and the norm of r, with the reduction
// order of rmsnorm_row_kernel: bit-identical to combine + add_rmsnorm.
template <typename TW>
__global__ void __launch_bounds__(kRowThreads) combine_add_rmsnorm_row_kernel(
    const __nv_bfloat16* __restrict__ y, const int32_t* __restrict__ slot_row, int K,
    const __nv_bfloat16* residual, __nv_bfloat16* residual_out, const TW* __restrict__ w,
    __nv_bfloat16* __restrict__ out, int hidden, float eps) {
  __shared__ float red[kRowThreads / 32];
  pdl_launch_dependents();
  pdl_wait();
  const long long row = blockIdx.x;
  const int nchunk = hidden >> 3;
  float v[kRowChunks][8], wv[kRowChunks][8], r[kRowChunks][8];
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
      load8(w + c * 8, wv[i]);
      load8(residual + row * hidden + c * 8, r[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }
  // ascending k, as combine_kernel: 8 slots' row loads in flight per chunk
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c >= nchunk) continue;
    for (int k0 = 0; k0 < K; k0 += 8) {
      int rr[8];
      uint4 u[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) rr[q] = k0 + q < K ? slot_row[row * K + k0 + q] : -1;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (rr[q] >= 0) u[q] = *reinterpret_cast<const uint4*>(y + static_cast<long long>(rr[q]) * hidden + c * 8);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (rr[q] < 0) continue;
        const float2 a = unpack_bf16x2(u[q].x), b = unpack_bf16x2(u[q].y), cc = unpack_bf16x2(u[q].z),
                     d = unpack_bf16x2(u[q].w);
        v[i][0] = fmaf(1.f, a.x, v[i][0]);
        v[i][1] = fmaf(1.f, a.y, v[i][1]);
        v[i][2] = fmaf(1.f, b.x, v[i][2]);
        v[i][3] = fmaf(1.f, b.y, v[i][3]);
        v[i][4] = fmaf(1.f, cc.x, v[i][4]);
        v[i][5] = fmaf(1.f, cc.y, v[i][5]);
        v[i][6] = fmaf(1.f, d.x, v[i][6]);
        v[i][7] = fmaf(1.f, d.y, v[i][7]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
      round_bf16(v[i]);  // the block output h, bf16
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] += r[i][j];
      round_bf16(v[i]);  // the residual stream, bf16
      store8(residual_out + row * hidden + c * 8, v[i]);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(v[i][j], v[i][j], ss);
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int q = 0; q < kRowThreads / 32; ++q) ss += red[q];
  const float rinv = rsqrtf(ss / static_cast<float>(hidden) + eps);
#pragma unroll
  for (int i = 0; i < kRowChunks; ++i) {
    const int c = threadIdx.x + i * kRowThreads;
    if (c < nchunk) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = v[i][j] * rinv * wv[i][j];
      store8(out + row * hidden + c * 8, o);
    }
  }
}

constexpr long long kRowKernelMaxRows = 512;

template <typename TX, typename TW, typename TO, bool kRes>
cudaError_t launch_rms(const void* x, const void* res, void* res_out, const void* w, void* out, long long rows,
                       int hidden, float eps, cudaStream_t s) {
  if (rows <= kRowKernelMaxRows && hidden <= kRowChunks * 8 * kRowThreads) {
    return launch_pdl(rmsnorm_row_kernel<TX, TW, TO, kRes>, dim3(static_cast<unsigned>(rows)), dim3(kRowThreads), 0,
                      s, static_cast<const TX*>(x), static_cast<const TX*>(res), static_cast<TX*>(res_out),
                      static_cast<const TW*>(w), static_cast<TO*>(out), hidden, eps);
  }
  const int warps = 8;
  const long long blocks = (rows + warps - 1) / warps;
  if constexpr (std::is_same<TX, __nv_bfloat16>::value) {
    rmsnorm_bf16_kernel<TW, TO, kRes><<<static_cast<unsigned>(blocks), warps * 32, 0, s>>>(
        static_cast<const TX*>(x), static_cast<const TX*>(res), static_cast<TX*>(res_out),
        static_cast<const TW*>(w), static_cast<TO*>(out), rows, hidden, eps);
    return cudaGetLastError();
  }
  rmsnorm_kernel<TX, TW, TO, kRes><<<static_cast<unsigned>(blocks), warps * 32, 0, s>>>(
      static_cast<const TX*>(x), static_cast<const TX*>(res), static_cast<TX*>(res_out),
      static_cast<const TW*>(w), static_cast<TO*>(out), rows, hidden, eps);
  return cudaGetLastError();
}

}  // namespace

cudaError_t rmsnorm_launch(const void* x, int x_dtype, const void* w, int w_dtype, void* out, int out_dtype,
                           long long rows, int hidden, float eps, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  using bf = __nv_bfloat16;
#define NKI_RMS(TX, TW, TO) return launch_rms<TX, TW, TO, false>(x, nullptr, nullptr, w, out, rows, hidden, eps, s)
  if (x_dtype == kBF16 && w_dtype == kF32 && out_dtype == kBF16) NKI_RMS(bf, float, bf);
  if (x_dtype == kBF16 && w_dtype == kBF16 && out_dtype == kBF16) NKI_RMS(bf, bf, bf);
  if (x_dtype == kBF16 && w_dtype == kF32 && out_dtype == kF32) NKI_RMS(bf, float, float);
  if (x_dtype == kF32 && w_dtype == kF32 && out_dtype == kF32) NKI_RMS(float, float, float);
  if (x_dtype == kF32 && w_dtype == kF32 && out_dtype == kBF16) NKI_RMS(float, float, bf);
  if (x_dtype == kF32 && w_dtype == kBF16 && out_dtype == kF32) NKI_RMS(float, bf, float);
#undef NKI_RMS
  return cudaErrorInvalidValue;
}

bool combine_add_rmsnorm_supported(long long rows, int hidden) {
  return rows <= kRowKernelMaxRows && hidden % 8 == 0 && hidden <= kRowChunks * 8 * kRowThreads;
}

cudaError_t combine_add_rmsnorm_launch(const __nv_bfloat16* y, const int32_t* slot_row, int K,
                                       const __nv_bfloat16* residual, __nv_bfloat16* residual_out, const void* w,
                                       int w_dtype, __nv_bfloat16* out, long long rows, int hidden, float eps,
                                       cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (!combine_add_rmsnorm_supported(rows, hidden)) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>(rows)), block(kRowThreads);
  if (w_dtype == kF32)
    return launch_pdl(combine_add_rmsnorm_row_kernel<float>, grid, block, 0, s, y, slot_row, K, residual,
                      residual_out, static_cast<const float*>(w), out, hidden, eps);
  if (w_dtype == kBF16)
    return launch_pdl(combine_add_rmsnorm_row_kernel<__nv_bfloat16>, grid, block, 0, s, y, slot_row, K, residual,
                      residual_out, static_cast<const __nv_bfloat16*>(w), out, hidden, eps);
  return cudaErrorInvalidValue;
}

cudaError_t add_rmsnorm_launch(const void* x, const void* residual, void* residual_out, const void* w, int w_dtype,
                               void* out, long long rows, int hidden, float eps, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  using bf = __nv_bfloat16;
  if (w_dtype == kF32) return launch_rms<bf, float, bf, true>(x, residual, residual_out, w, out, rows, hidden, eps, s);
  if (w_dtype == kBF16) return launch_rms<bf, bf, bf, true>(x, residual, residual_out, w, out, rows, hidden, eps, s);
  return cudaErrorInvalidValue;
}

// ------------------------------------------------------------------ K6
// One warp per (token, head) for the q and k heads; v heads are copied when
// the output is a different buffer.  head_dim 128: lane l owns elements
// [4l, 4l+4); its rotate-half partner lives in lane l ^ 16.
namespace {

// One warp per token: the RoPE cos / sin of the lane's 4 elements are computed
// once (powf + sincosf are the kernel's costly part) and serve all the
// token's q and k heads; heads are loaded kAhead at a time so their loads are
// in flight together.  Each head's arithmetic is norm_rope_head128's.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const __nv_bfloat16* in, __nv_bfloat16* out, const void* qw,
                                                           const void* kw, int w_dtype,
                                                           const long long* __restrict__ positions, long long tokens,
                                                           int n_heads, int n_kv, float theta, float eps) {
  constexpr int D = kHeadDim;
  constexpr int kAhead = 4;
  const int lane = threadIdx.x & 31;
  const int heads_total = n_heads + 2 * n_kv;
  const long long t = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const long long row = t * heads_total * D + lane * 4;
  float cs[4], sn[4];
  rope_cs_lane(static_cast<float>(positions[t]), theta, lane, cs, sn);
  for (int h0 = 0; h0 < heads_total; h0 += kAhead) {
    uint2 raw[kAhead];
#pragma unroll
    for (int a = 0; a < kAhead; ++a)
      if (h0 + a < heads_total) raw[a] = *reinterpret_cast<const uint2*>(in + row + static_cast<long long>(h0 + a) * D);
#pragma unroll
    for (int a = 0; a < kAhead; ++a) {
      const int h = h0 + a;
      if (h >= heads_total) break;
      __nv_bfloat16* dst = out + row + static_cast<long long>(h) * D;
      if (h >= n_heads + n_kv) {  // V head: pass through
        if (in != out) *reinterpret_cast<uint2*>(dst) = raw[a];
        continue;
      }
      const float2 x0 = unpack_bf16x2(raw[a].x), x1 = unpack_bf16x2(raw[a].y);
      const float v[4] = {x0.x, x0.y, x1.x, x1.y};
      float o[4];
      norm_rope_head128_cs(v, h < n_heads ? qw : kw, w_dtype, eps, lane, cs, sn, o);
      head_store4(dst, o);
    }
  }
}

}  // namespace

cudaError_t qk_norm_rope_launch(const void* qkv_in, void* qkv_out, const void* qw, const void* kw, int w_dtype,
                                const long long* positions, long long tokens, int n_heads, int n_kv, int head_dim,
                                float theta, float eps, cudaStream_t s) {
  if (tokens == 0) return cudaSuccess;
  if (head_dim != 128) return cudaErrorInvalidValue;
  const int wpb = 8;  // one warp per token
  const long long blocks = (tokens + wpb - 1) / wpb;
  qk_norm_rope_kernel<<<static_cast<unsigned>(blocks), wpb * 32, 0, s>>>(
      static_cast<const __nv_bfloat16*>(qkv_in), static_cast<__nv_bfloat16*>(qkv_out), qw, kw, w_dtype, positions,
      tokens, n_heads, n_kv, theta, eps);
  return cudaGetLastError();
}

}  // namespace nkimoe
