// nkimoe_moe_block_noalloc: the whole MoE block for callers that cannot
// allocate GPU memory.
//
// Some callers cannot call cudaMalloc or hand this library a workspace: an
// inference server that has reserved all device memory for its KV cache and
// weights up front, a host runtime whose allocator may not be entered from the
// thread that issues the layer (or only at start-up), or an embedding that
// forbids allocation once its CUDA graphs are being recorded.  For them this
// entry point runs nkimoe_moe_block on a fixed scratch array that is part of
// the library image: a file-scope __device__ array of kNoAllocScratchBytes
// that every GPU which loads the library holds until the process exits.  The
// call itself allocates nothing.
//
// The array's name is only a host-side stand-in in host code; its device
// address is obtained once per device with cudaGetSymbolAddress, with that
// device current, on the first call made on that device.  Make that first call
// before any stream capture.
#include <cstdio>
#include <mutex>

#include "kernels.h"
#include "nkimoe.h"

namespace nkimoe {
namespace {

constexpr size_t kNoAllocScratchBytes = NKIMOE_NOALLOC_SCRATCH_BYTES;  // 8 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on the
// first call per device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) return NKIMOE_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return NKIMOE_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return NKIMOE_OK;
}

}  // namespace
}  // namespace nkimoe

extern "C" {

int nkimoe_moe_block_noalloc(const void* x, const float* router_w, const float* router_bias,
                             const void* router_w_split, const void* w13, const void* w2, void* out,
                             int32_t* topk_idx_out, float* topk_w_out, int64_t T, int64_t H, int64_t I, int64_t E,
                             int64_t K, void* stream) {
  // shapes first: a negative T would otherwise show up as a huge scratch need
  const int rc = nkimoe::check_moe_shapes(T, H, I, E, K);
  if (rc != NKIMOE_OK) return rc;
  const size_t need = nkimoe_moe_workspace_bytes(T, H, I, E, K);
  if (need > nkimoe::kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "nkimoe_moe_block_noalloc: %lld tokens need %zu scratch bytes, more than its fixed %zu; "
             "use nkimoe_moe_block with a workspace",
             static_cast<long long>(T), need, nkimoe::kNoAllocScratchBytes);
    nkimoe::set_last_error(msg);
    return NKIMOE_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  if (nkimoe::noalloc_scratch(&scratch) != NKIMOE_OK) {
    nkimoe::set_last_error("nkimoe_moe_block_noalloc: cudaGetSymbolAddress of the scratch array failed");
    return NKIMOE_ERR_CUDA;
  }
  return nkimoe_moe_block(x, router_w, router_bias, router_w_split, w13, w2, out, topk_idx_out, topk_w_out, T, H, I,
                          E, K, scratch, nkimoe::kNoAllocScratchBytes, stream);
}

// The device status word of the no-allocation entry point sits at the start of
// the library's scratch array, which its callers cannot name: this reads and
// clears it for them, as nkimoe_read_status does for a workspace.
int nkimoe_noalloc_read_status(void* stream, int* status_out) {
  void* scratch = nullptr;
  if (nkimoe::noalloc_scratch(&scratch) != NKIMOE_OK) {
    nkimoe::set_last_error("nkimoe_noalloc_read_status: cudaGetSymbolAddress of the scratch array failed");
    return NKIMOE_ERR_CUDA;
  }
  return nkimoe_read_status(scratch, stream, status_out);
}

}  // extern "C"
