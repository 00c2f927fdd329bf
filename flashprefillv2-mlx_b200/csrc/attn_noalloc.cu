// fpv2_sparse_attention_noalloc: the sparse-attention entry point for callers
// that cannot allocate device memory.
//
// Some callers of this library cannot hand it even a few bytes of workspace:
// serving engines that reserve nearly all HBM for their KV-cache pool at start
// up and forbid any allocation outside it, and pipelines where a cudaMalloc
// (which may synchronise the device) is not allowed between asynchronous
// launches. This variant therefore keeps the attention kernel's only scratch --
// its work-queue counter -- in a fixed array compiled into the library, so the
// caller passes inputs and outputs and nothing else.
//
// Limits and sharing:
// * the array is FPV2_NOALLOC_SCRATCH_BYTES (256 bytes) on every GPU that loads
//   the library and stays allocated until the process exits;
// * every call on a device uses the same array: it is cleared on the caller's
//   stream before each launch, and calls whose launches overlap on the GPU (for
//   example on two streams) race on it;
// * the first call on a device looks up the array's device address
//   (cudaGetSymbolAddress with that device current); make that first call
//   before any stream capture. The address is cached for the life of the
//   process, so the library must not be used across a cudaDeviceReset of that
//   device (the array is re-created at a new address);
// * with only this scratch the call runs without the fp16 copy of V and the
//   split of long work items that a full caller workspace enables.
#include <mutex>

#include "../../include/fpv2_b200.h"
#include "common.cuh"

namespace fpv2 {

int report_error(int code, const char* msg);   // capi.cu

namespace {

constexpr int kNoAllocScratchBytes = FPV2_NOALLOC_SCRATCH_BYTES;
static_assert(FPV2_ATTN_WORKSPACE_BYTES <= kNoAllocScratchBytes,
              "the attention workspace must fit the static scratch array");

// The scratch itself. Host code must not pass this name to a kernel: on the
// host it is only a stand-in symbol; its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device (set up once per device).
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess)
    return report_error(FPV2_ERR_CUDA, "cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return report_error(FPV2_ERR_UNSUPPORTED, "device index");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return report_error(FPV2_ERR_CUDA, "cudaGetSymbolAddress of the no-alloc scratch failed");
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return FPV2_OK;
}

}  // namespace

}  // namespace fpv2

extern "C" int fpv2_sparse_attention_noalloc(
    const void* q, const void* k, const void* v, const void* pooled_k, const void* pooled_v,
    int pooled_dtype, const int32_t* selected_ids, const int32_t* selected_counts,
    const int32_t* pruned_ids, const int32_t* pruned_counts, int dtype, int32_t q_heads,
    int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len, int32_t head_dim,
    int32_t offset, int32_t query_length, int32_t key_length, float scale, int32_t block_k,
    int32_t tile_q, int32_t mean_correction, void* out, void* stream) {
  // The scratch holds one work-queue counter; the counter indexes work items
  // (128-row chunks of the selection tiles), so the problem size is limited to
  // FPV2_NOALLOC_MAX_WORK_ITEMS of them.
  if (kv_heads > 0 && tile_q > 0 && padded_q_len > 0 && q_heads > 0) {
    const long long rows = (long long)(q_heads / kv_heads) * tile_q;
    const long long items = (long long)kv_heads * (padded_q_len / tile_q) * ((rows + 127) / 128);
    if (items > FPV2_NOALLOC_MAX_WORK_ITEMS)
      return fpv2::report_error(FPV2_ERR_INVALID_ARGUMENT,
                                "problem too large for the no-alloc scratch: more than "
                                "FPV2_NOALLOC_MAX_WORK_ITEMS work items");
  }
  void* scratch = nullptr;
  const int rc = fpv2::scratch_address(&scratch);
  if (rc != FPV2_OK) return rc;
  return fpv2_sparse_attention(q, k, v, pooled_k, pooled_v, pooled_dtype, selected_ids,
                               selected_counts, pruned_ids, pruned_counts, dtype, q_heads,
                               kv_heads, padded_q_len, padded_k_len, head_dim, offset,
                               query_length, key_length, scale, block_k, tile_q, mean_correction,
                               out, scratch, fpv2::kNoAllocScratchBytes, stream);
}
