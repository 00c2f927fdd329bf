// C ABI of the FPV2 B200 path (declared in include/fpv2_b200.h).
//
// Each entry point checks its scalars and pointers, picks the tcgen05 kernel
// when the shape fits it and the generic CUDA-core kernel otherwise, and
// enqueues on the caller's stream. No host synchronisation, no allocation.
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "../../include/fpv2_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fpv2 {

// Status word read by fpv2_device_status; one copy per device context.
__device__ int g_device_status;

namespace {

thread_local std::string t_last_error;
double g_wait_budget_ms = 2000.0;

struct DeviceInfo {
  bool ready = false;
  int* status = nullptr;
  int num_sms = 0;
  int clock_khz = 0;
  int major = 0;
};
constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::mutex g_mutex;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(FPV2_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

// Per-device set-up with that device current: address of the status word,
// SM count and clock (for the clock64 wait budget).
int device_info(DeviceInfo** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FPV2_ERR_UNSUPPORTED, "device index %d", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceInfo& d = g_devices[dev];
  if (!d.ready) {
    e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&d.clock_khz, cudaDevAttrClockRate, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), g_device_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    d.ready = true;
  }
  if (d.major != 10)
    return fail(FPV2_ERR_UNSUPPORTED, "this build targets sm_100a; device %d is sm_%d", dev,
                d.major * 10);
  *out = &d;
  return FPV2_OK;
}

TcLaunch tc_launch(const DeviceInfo& d) {
  TcLaunch L;
  L.status = d.status;
  const double khz = d.clock_khz > 0 ? (double)d.clock_khz : 2.0e6;
  // clock64 counts SM cycles; budget in cycles at the highest clock.
  L.budget = (long long)(g_wait_budget_ms * khz);
  if (L.budget < 1000) L.budget = 1000;
  L.num_sms = d.num_sms;
  return L;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool valid_dtype(int dt) { return dt == DT_F16 || dt == DT_BF16 || dt == DT_F32; }
size_t dt_size(int dt) { return dt == DT_F32 ? 4 : 2; }

}  // namespace

// Record `msg` as the calling thread's last error and return `code` (for entry
// points defined in other translation units).
int report_error(int code, const char* msg) {
  t_last_error = msg;
  return code;
}

bool encode_tmap_3d(CUtensorMap* map, const void* base, int dt, uint64_t d0, uint64_t d1,
                    uint64_t d2, uint32_t b0, uint32_t b1, uint32_t b2) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const size_t es = dt_size(dt);
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {d0 * es, d0 * d1 * es};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType ty = dt == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dt == DT_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = fn(map, ty, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_tmap_pages(CUtensorMap* map, const void* base, int dt, uint64_t D, uint64_t heads,
                       uint64_t page_size, uint64_t pages, uint32_t rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return false;
  const size_t es = dt_size(dt);
  cuuint64_t dims[4] = {D, heads, page_size, pages};
  cuuint64_t strides[3] = {D * es, heads * D * es, page_size * heads * D * es};
  cuuint32_t box[4] = {64, 1, rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType ty = dt == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, ty, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Shared validation of the selection geometry (fpv2/selection.py:83-106).
static int check_select_geom(const SelectGeom& g) {
  if (g.Hkv <= 0 || g.Hq <= 0 || g.Hq % g.Hkv)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "query heads must be divisible by KV heads");
  if (g.D <= 0) return fail(FPV2_ERR_INVALID_ARGUMENT, "head_dim must be positive");
  if (g.block_k <= 0 || g.tile_q <= 0)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "block_k and tile_q must be positive");
  if (g.Lq_pad <= 0 || g.Lq_pad % g.tile_q)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "query length must be padded to a multiple of tile_q");
  if (!(0 < g.valid_lq && g.valid_lq <= g.Lq_pad))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "query_length must be in (0, padded_q_len]");
  if (g.offset < 0) return fail(FPV2_ERR_INVALID_ARGUMENT, "offset must be non-negative");
  if (g.Nb <= 0) return fail(FPV2_ERR_INVALID_ARGUMENT, "num_blocks must be positive");
  if ((long long)g.offset + g.valid_lq > (long long)g.Nb * g.block_k)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "queries extend beyond the represented key sequence");
  if (g.alpha < 0.f) return fail(FPV2_ERR_INVALID_ARGUMENT, "alpha must be non-negative");
  if (g.sink < 0 || g.window < 0)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "sink_tokens and window_tokens must be non-negative");
  if (g.last_n < 0) return fail(FPV2_ERR_INVALID_ARGUMENT, "last_n_blocks must be non-negative");
  return FPV2_OK;
}

// Selection with lists and/or mask: tcgen05 kernel when the shape fits. float32
// pooled keys with 16-bit queries run on it too when the workspace holds their
// three 16-bit parts; otherwise (and for float32 queries) on the CUDA cores.
static int run_select(const SelectGeom& g, const void* q, int q_dt, const void* pk, int pk_dt,
                      uint8_t* mask, const SelectLists& lists, const DeviceInfo& d,
                      void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  cudaError_t e;
  const bool aligned = (reinterpret_cast<uintptr_t>(q) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(pk) % 16 == 0);
  int nparts = 1;
  const int* k_exp = nullptr;
  if (pk_dt == DT_F32 && q_dt != DT_F32 && aligned && select_tc_supported(g, q_dt) &&
      workspace != nullptr && reinterpret_cast<uintptr_t>(workspace) % 256 == 0 &&
      workspace_bytes >= (int64_t)pk_split3_bytes(g.Hkv, g.Nb, g.D)) {
    e = launch_pk_split3(reinterpret_cast<const float*>(pk), workspace, q_dt, g.Hkv, g.Nb, g.D,
                         &k_exp, stream);
    if (e != cudaSuccess) return cuda_fail(e, "pooled-key split launch");
    pk = workspace;
    pk_dt = q_dt;
    nparts = 3;
  }
  if (q_dt == pk_dt && aligned && select_tc_supported(g, q_dt)) {
    SelectTcArgs a;
    a.nparts = nparts;
    a.k_exp = k_exp;
    a.g = g;
    const int R = g.G * g.tile_q;
    a.NC = R < 128 ? R : 128;
    a.box_rows = g.tile_q < a.NC ? g.tile_q : a.NC;
    a.box_heads = a.NC / a.box_rows;
    a.dt = q_dt;
    a.mask = mask;
    a.sel_ids = lists.sel_ids;
    a.sel_counts = lists.sel_counts;
    a.pr_ids = lists.pr_ids;
    a.pr_counts = lists.pr_counts;
    e = launch_select_tc(a, q, pk, tc_launch(d), stream);
    if (e != cudaSuccess) return cuda_fail(e, "select_tc launch");
    return FPV2_OK;
  }
  e = launch_select_generic(g, q, q_dt, pk, pk_dt, mask, lists, stream);
  if (e != cudaSuccess) return cuda_fail(e, "select_generic launch");
  return FPV2_OK;
}

std::atomic<long long> g_launch_count{0};

void count_launch() { g_launch_count.fetch_add(1, std::memory_order_relaxed); }

}  // namespace fpv2

using namespace fpv2;

extern "C" {

int fpv2_version(void) { return 100; }

int64_t fpv2_launch_count(void) { return g_launch_count.load(std::memory_order_relaxed); }

const char* fpv2_last_error(void) { return t_last_error.c_str(); }

int fpv2_device_supported(int device) {
  int major = 0;
  cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
  if (major != 10)
    return fail(FPV2_ERR_UNSUPPORTED, "device %d is sm_%d; this build targets sm_100a", device,
                major * 10);
  return FPV2_OK;
}

int fpv2_set_wait_budget_ms(double milliseconds) {
  if (!(milliseconds > 0.0)) return fail(FPV2_ERR_INVALID_ARGUMENT, "budget must be positive");
  g_wait_budget_ms = milliseconds;
  return FPV2_OK;
}

int fpv2_device_status(void* stream, int clear, int32_t* status_out) {
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  int v = 0;
  e = cudaMemcpy(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  if (clear) {
    e = cudaMemset(d->status, 0, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clear status");
  }
  if (status_out) *status_out = v;
  return FPV2_OK;
}

int fpv2_pool_blocks(const void* x, int x_dtype, int64_t heads, int64_t length,
                     int32_t head_dim, int32_t block_size, void* out, int out_dtype,
                     void* stream) {
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (block_size <= 0) return fail(FPV2_ERR_INVALID_ARGUMENT, "block_size must be positive");
  if (heads < 0 || length < 0 || head_dim <= 0)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "invalid shape");
  if (length % block_size)
    return fail(FPV2_ERR_INVALID_ARGUMENT,
                "sequence length %lld must be divisible by block_size %d", (long long)length,
                block_size);
  if (heads * length > 0 && (x == nullptr || out == nullptr))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "null tensor pointer");
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  PoolArgs a;
  a.x[0] = x;
  a.x[1] = nullptr;
  a.out[0] = out;
  a.out[1] = nullptr;
  a.heads = heads;
  a.length = length;
  a.D = head_dim;
  a.bs = block_size;
  cudaError_t e = launch_pool(a, 1, x_dtype, out_dtype, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pool launch");
  return FPV2_OK;
}

int fpv2_block_select(const void* q, int q_dtype, const void* pooled_k, int k_dtype,
                      int32_t q_heads, int32_t kv_heads, int32_t padded_q_len,
                      int32_t num_blocks, int32_t head_dim, int32_t offset,
                      int32_t query_length, float scale, int32_t block_k, int32_t tile_q,
                      float alpha, int32_t sink_tokens, int32_t window_tokens,
                      int32_t last_n_blocks, uint8_t* selected, float* raw_scores,
                      void* workspace, int64_t workspace_bytes, void* stream) {
  if (!valid_dtype(q_dtype) || !valid_dtype(k_dtype))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "unknown dtype code");
  SelectGeom g;
  g.Hq = q_heads;
  g.Hkv = kv_heads;
  g.G = kv_heads > 0 ? q_heads / kv_heads : 0;
  g.Lq_pad = padded_q_len;
  g.Nb = num_blocks;
  g.D = head_dim;
  g.Nt = tile_q > 0 ? padded_q_len / tile_q : 0;
  g.offset = offset;
  g.valid_lq = query_length;
  g.valid_lk = num_blocks * block_k;
  g.block_k = block_k;
  g.tile_q = tile_q;
  g.sink = sink_tokens;
  g.window = window_tokens;
  g.last_n = last_n_blocks;
  g.scale = scale;
  g.alpha = alpha;
  int rc = check_select_geom(g);
  if (rc != FPV2_OK) return rc;
  if (q == nullptr || pooled_k == nullptr || selected == nullptr)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "null tensor pointer");
  DeviceInfo* d = nullptr;
  rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SelectLists none{nullptr, nullptr, nullptr, nullptr};
  rc = run_select(g, q, q_dtype, pooled_k, k_dtype, selected, none, *d, workspace, workspace_bytes, s);
  if (rc != FPV2_OK) return rc;
  if (raw_scores != nullptr) {
    cudaError_t e = launch_raw_scores(g, q, q_dtype, pooled_k, k_dtype, raw_scores, s);
    if (e != cudaSuccess) return cuda_fail(e, "raw scores launch");
  }
  return FPV2_OK;
}

int fpv2_compact_block_indices(const uint8_t* selected, int32_t kv_heads, int32_t num_tiles,
                               int32_t num_blocks, int32_t block_k, int32_t tile_q,
                               int32_t offset, int32_t query_length, int32_t key_length,
                               int32_t* selected_ids, int32_t* selected_counts,
                               int32_t* pruned_ids, int32_t* pruned_counts, void* stream) {
  if (kv_heads < 0 || num_tiles < 0 || num_blocks <= 0 || block_k <= 0 || tile_q <= 0)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "invalid shape");
  if (offset < 0) return fail(FPV2_ERR_INVALID_ARGUMENT, "offset must be non-negative");
  const long long pq = (long long)num_tiles * tile_q;
  const long long rk = (long long)num_blocks * block_k;
  if (!(0 < query_length && query_length <= pq))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "query_length is inconsistent with selected tiles");
  if (!(0 < key_length && key_length <= rk))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "key_length is inconsistent with selected blocks");
  if ((long long)offset + query_length > key_length)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "queries extend beyond key_length");
  if (!selected || !selected_ids || !selected_counts || !pruned_ids || !pruned_counts)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "null tensor pointer");
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  cudaError_t e = launch_compact(selected, kv_heads, num_tiles, num_blocks, block_k, tile_q,
                                 offset, key_length, selected_ids, selected_counts, pruned_ids,
                                 pruned_counts, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "compact launch");
  return FPV2_OK;
}

int fpv2_index_stage(const void* q, const void* k, const void* v, int dtype,
                     int32_t q_heads, int32_t kv_heads, int32_t padded_q_len,
                     int32_t padded_k_len, int32_t head_dim, int32_t offset,
                     int32_t query_length, int32_t key_length, float scale,
                     int32_t block_k, int32_t tile_q, float alpha, int32_t sink_tokens,
                     int32_t window_tokens, int32_t last_n_blocks, int pooled_dtype,
                     void* pooled_k, void* pooled_v, int32_t* selected_ids,
                     int32_t* selected_counts, int32_t* pruned_ids, int32_t* pruned_counts,
                     uint8_t* selected, void* workspace, int64_t workspace_bytes, void* stream) {
  if (dtype != DT_F16 && dtype != DT_BF16 && dtype != DT_F32)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (pooled_dtype != dtype && pooled_dtype != DT_F32)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "pooled_dtype must be the input dtype or FPV2_F32");
  if (block_k <= 0 || padded_k_len <= 0 || padded_k_len % block_k)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "k/v length must be a positive multiple of block_k");
  SelectGeom g;
  g.Hq = q_heads;
  g.Hkv = kv_heads;
  g.G = kv_heads > 0 ? q_heads / kv_heads : 0;
  g.Lq_pad = padded_q_len;
  g.Nb = padded_k_len / block_k;
  g.D = head_dim;
  g.Nt = tile_q > 0 ? padded_q_len / tile_q : 0;
  g.offset = offset;
  g.valid_lq = query_length;
  g.valid_lk = key_length;
  g.block_k = block_k;
  g.tile_q = tile_q;
  g.sink = sink_tokens;
  g.window = window_tokens;
  g.last_n = last_n_blocks;
  g.scale = scale;
  g.alpha = alpha;
  int rc = check_select_geom(g);
  if (rc != FPV2_OK) return rc;
  if (!(0 < key_length && key_length <= padded_k_len))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "key_length must fit within padded k/v");
  if ((long long)offset + query_length > key_length)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "queries extend beyond key_length");
  if (!q || !k || !v || !pooled_k || !pooled_v || !selected_ids || !selected_counts ||
      !pruned_ids || !pruned_counts)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "null tensor pointer");
  DeviceInfo* d = nullptr;
  rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  PoolArgs pa;
  pa.x[0] = k;
  pa.x[1] = v;
  pa.out[0] = pooled_k;
  pa.out[1] = pooled_v;
  pa.heads = kv_heads;
  pa.length = padded_k_len;
  pa.D = head_dim;
  pa.bs = block_k;
  cudaError_t e = launch_pool(pa, 2, dtype, pooled_dtype, s);
  if (e != cudaSuccess) return cuda_fail(e, "pool launch");
  SelectLists lists{selected_ids, selected_counts, pruned_ids, pruned_counts};
  return run_select(g, q, dtype, pooled_k, pooled_dtype, selected, lists, *d, workspace,
                    workspace_bytes, s);
}

int64_t fpv2_select_workspace_bytes(int q_dtype, int k_dtype, int32_t kv_heads,
                                    int32_t num_blocks, int32_t head_dim) {
  if (k_dtype != DT_F32 || (q_dtype != DT_BF16 && q_dtype != DT_F16) || kv_heads <= 0 ||
      num_blocks <= 0 || head_dim <= 0)
    return 0;
  return (int64_t)pk_split3_bytes(kv_heads, num_blocks, head_dim);
}

namespace fpv2 {
namespace {

// Shared body of fpv2_sparse_attention and fpv2_sparse_attention_multicast.
// K/V in page pools (fpv2_sparse_attention_paged); null for contiguous K/V.
struct PagedKV {
  const int32_t* table;
  int32_t table_len, num_pages, page_size;
};

int run_sparse_attention(const void* q, const void* k, const void* v, const void* pooled_k,
                         const void* pooled_v, int pooled_dtype, const int32_t* selected_ids,
                         const int32_t* selected_counts, const int32_t* pruned_ids,
                         const int32_t* pruned_counts, int dtype, int32_t q_heads,
                         int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len,
                         int32_t head_dim, int32_t offset, int32_t query_length,
                         int32_t key_length, float scale, int32_t block_k, int32_t tile_q,
                         int32_t mean_correction, void* out, void* out_mc, int32_t head_offset,
                         int32_t heads_total, void* workspace, int64_t workspace_bytes,
                         void* stream, const PagedKV* paged = nullptr) {
  if (dtype != DT_F16 && dtype != DT_BF16)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "q, k, and v must share float16 or bfloat16 dtype");
  if (pooled_dtype != dtype && pooled_dtype != DT_F32)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "pooled_dtype must be the input dtype or FPV2_F32");
  if (kv_heads <= 0 || q_heads <= 0 || q_heads % kv_heads)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "query heads must be divisible by KV heads");
  if (head_dim <= 0 || head_dim > 256)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "head dimension must be in [1, 256]");
  if (block_k <= 0 || tile_q <= 0 || padded_q_len <= 0 || padded_k_len <= 0 ||
      padded_q_len % tile_q || padded_k_len % block_k)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "q and k/v sequence lengths must be tile/block aligned");
  if (!(0 < query_length && query_length <= padded_q_len))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "query_length must fit within padded q");
  if (!(0 < key_length && key_length <= padded_k_len))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "key_length must fit within padded k/v");
  if (offset < 0 || (long long)offset + query_length > key_length)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "offset does not align queries within the key sequence");
  if (!q || !k || !v || (!out && !out_mc) || !selected_ids || !selected_counts ||
      (mean_correction && (!pooled_k || !pooled_v || !pruned_ids || !pruned_counts)))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (out_mc != nullptr &&
      (head_offset < 0 || heads_total < q_heads || head_offset > heads_total - q_heads))
    return fail(FPV2_ERR_INVALID_ARGUMENT, "multicast output heads out of range");
  if (paged != nullptr) {
    if (paged->table == nullptr || paged->page_size <= 0 || paged->num_pages <= 0 ||
        paged->table_len <= 0)
      return fail(FPV2_ERR_INVALID_ARGUMENT, "paged K/V needs a block table, pages and a page size");
    if ((long long)paged->table_len * paged->page_size < padded_k_len)
      return fail(FPV2_ERR_INVALID_ARGUMENT, "block table does not cover the padded key length");
  }
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  AttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.pk = pooled_k;
  a.pv = pooled_v;
  a.pooled_dt = pooled_dtype;
  a.sel_ids = selected_ids;
  a.sel_counts = selected_counts;
  a.pr_ids = pruned_ids;
  a.pr_counts = pruned_counts;
  a.out = out;
  a.dt = dtype;
  a.Hq = q_heads;
  a.Hkv = kv_heads;
  a.G = q_heads / kv_heads;
  a.Lq_pad = padded_q_len;
  a.Lk_pad = padded_k_len;
  a.D = head_dim;
  a.Nt = padded_q_len / tile_q;
  a.Nb = padded_k_len / block_k;
  a.offset = offset;
  a.valid_lq = query_length;
  a.valid_lk = key_length;
  a.block_k = block_k;
  a.tile_q = tile_q;
  a.corr = mean_correction ? 1 : 0;
  a.scale_log2 = scale * kLog2e;
  a.corr_shift = (float)log2((double)block_k);
  a.out_mc = out_mc;
  a.status = d->status;
  a.mc_head_offset = head_offset;
  a.mc_heads = heads_total;
  if (paged != nullptr) {
    a.block_table = paged->table;
    a.page_size = paged->page_size;
    a.num_pages = paged->num_pages;
    a.table_len = paged->table_len;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool aligned = reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(k) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(v) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(out_mc) % 16 == 0 &&
                       (!a.corr || (reinterpret_cast<uintptr_t>(pooled_k) % 16 == 0 &&
                                    reinterpret_cast<uintptr_t>(pooled_v) % 16 == 0));
  cudaError_t e;
  const bool use_tc = aligned && attn_tc_supported(a);
  const bool use_wide = !use_tc && aligned && attn_wide_supported(a);
  // bf16 inputs with room in the workspace: P.V in fp16 on an exact fp16 copy of V
  // (the copy and its scratch lead the workspace; the rest serves the kernel).
  if ((use_tc || use_wide) && dtype == DT_BF16 && workspace != nullptr &&
      reinterpret_cast<uintptr_t>(workspace) % 256 == 0) {
    const size_t conv = v_conv_bytes(kv_heads, padded_k_len, head_dim, a.Nb);
    if (workspace_bytes >= (int64_t)(conv + kAttnMinWorkspace)) {
      char* base = reinterpret_cast<char*>(workspace);
      const size_t v_bytes = ((size_t)kv_heads * padded_k_len * head_dim * 2 + 255) / 256 * 256;
      const size_t pv_bytes = ((size_t)kv_heads * a.Nb * head_dim * 2 + 255) / 256 * 256;
      VConvArgs c;
      c.v = v;
      c.table = paged != nullptr ? paged->table : nullptr;
      c.table_len = paged != nullptr ? paged->table_len : 0;
      c.num_pages = paged != nullptr ? paged->num_pages : 0;
      c.page_size = paged != nullptr ? paged->page_size : 0;
      c.Hkv = kv_heads;
      c.L = padded_k_len;
      c.D = head_dim;
      c.pv = (a.corr && pooled_dtype == dtype) ? pooled_v : nullptr;
      c.Nb = a.Nb;
      c.v16 = base;
      c.pv16 = base + v_bytes;
      c.v_exp = reinterpret_cast<int*>(base + v_bytes + pv_bytes);
      c.absmax = reinterpret_cast<unsigned*>(c.v_exp + kv_heads);
      e = launch_v_to_f16(c, s);
      if (e != cudaSuccess) return cuda_fail(e, "V conversion launch");
      a.vdt = DT_F16;
      a.v_conv = c.v16;
      a.pv_conv = c.pv != nullptr ? c.pv16 : nullptr;
      a.v_exp = c.v_exp;
      workspace = base + conv;
      workspace_bytes -= (int64_t)conv;
    }
  }
  if (use_tc) {
    const bool ws_ok = workspace != nullptr && reinterpret_cast<uintptr_t>(workspace) % 4 == 0;
    e = launch_attn_tc(a, tc_launch(*d), ws_ok ? workspace : nullptr, ws_ok ? workspace_bytes : 0, s);
    if (e != cudaSuccess) return cuda_fail(e, "attn_tc launch");
  } else if (use_wide) {
    int* sched = (workspace != nullptr && workspace_bytes >= (int64_t)sizeof(int))
                     ? reinterpret_cast<int*>(workspace)
                     : nullptr;
    e = launch_attn_wide(a, tc_launch(*d), sched, s);
    if (e != cudaSuccess) return cuda_fail(e, "attn_wide launch");
  } else if (paged != nullptr) {
    return fail(FPV2_ERR_UNSUPPORTED,
                "paged K/V needs the tcgen05 path (bf16/fp16, head_dim 64/96/128, aligned, block_k a "
                "multiple of 128, page_size a multiple of 8 that divides 128 or is a multiple of 128)");
  } else if (out_mc != nullptr) {
    return fail(FPV2_ERR_UNSUPPORTED,
                "multicast output needs the tcgen05 path (bf16/fp16, head_dim 64/96/128/256, aligned)");
  } else {
    e = launch_attn_generic(a, s);
    if (e != cudaSuccess) return cuda_fail(e, "attn_generic launch");
  }
  return FPV2_OK;
}

}  // namespace
}  // namespace fpv2

int fpv2_sparse_attention(const void* q, const void* k, const void* v, const void* pooled_k,
                          const void* pooled_v, int pooled_dtype,
                          const int32_t* selected_ids, const int32_t* selected_counts,
                          const int32_t* pruned_ids, const int32_t* pruned_counts, int dtype,
                          int32_t q_heads, int32_t kv_heads, int32_t padded_q_len,
                          int32_t padded_k_len, int32_t head_dim, int32_t offset,
                          int32_t query_length, int32_t key_length, float scale,
                          int32_t block_k, int32_t tile_q, int32_t mean_correction,
                          void* out, void* workspace, int64_t workspace_bytes,
                          void* stream) {
  return fpv2::run_sparse_attention(q, k, v, pooled_k, pooled_v, pooled_dtype, selected_ids,
                                    selected_counts, pruned_ids, pruned_counts, dtype, q_heads,
                                    kv_heads, padded_q_len, padded_k_len, head_dim, offset,
                                    query_length, key_length, scale, block_k, tile_q,
                                    mean_correction, out, nullptr, 0, 0, workspace,
                                    workspace_bytes, stream);
}

int64_t fpv2_attention_workspace_bytes(int dtype, int32_t q_heads, int32_t kv_heads,
                                       int32_t padded_q_len, int32_t padded_k_len,
                                       int32_t head_dim, int32_t block_k, int32_t tile_q,
                                       int pooled_dtype, int32_t mean_correction) {
  if (kv_heads <= 0 || q_heads <= 0 || q_heads % kv_heads || tile_q <= 0 || block_k <= 0 ||
      padded_q_len <= 0 || padded_k_len <= 0 || padded_q_len % tile_q || padded_k_len % block_k)
    return FPV2_ATTN_WORKSPACE_BYTES;
  AttnArgs a;
  a.dt = dtype;
  a.pooled_dt = pooled_dtype;
  a.Hq = q_heads;
  a.Hkv = kv_heads;
  a.G = q_heads / kv_heads;
  a.Lq_pad = padded_q_len;
  a.Lk_pad = padded_k_len;
  a.D = head_dim;
  a.Nt = padded_q_len / tile_q;
  a.Nb = padded_k_len / block_k;
  a.block_k = block_k;
  a.tile_q = tile_q;
  a.corr = mean_correction ? 1 : 0;
  a.scale_log2 = 1.f;
  size_t bytes = attn_tc_workspace_bytes(a);
  if (dtype == DT_BF16 && (attn_tc_supported(a) || attn_wide_supported(a)))
    bytes += v_conv_bytes(kv_heads, padded_k_len, head_dim, a.Nb);   // fp16 copy of V
  return (int64_t)std::max<size_t>(bytes, FPV2_ATTN_WORKSPACE_BYTES);
}

int fpv2_sparse_attention_multicast(
    const void* q, const void* k, const void* v, const void* pooled_k, const void* pooled_v,
    int pooled_dtype, const int32_t* selected_ids, const int32_t* selected_counts,
    const int32_t* pruned_ids, const int32_t* pruned_counts, int dtype, int32_t q_heads,
    int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len, int32_t head_dim,
    int32_t offset, int32_t query_length, int32_t key_length, float scale, int32_t block_k,
    int32_t tile_q, int32_t mean_correction, void* out_multicast, int32_t head_offset,
    int32_t heads_total, void* workspace, int64_t workspace_bytes, void* stream) {
  if (out_multicast == nullptr) return fail(FPV2_ERR_INVALID_ARGUMENT, "null multicast output");
  return fpv2::run_sparse_attention(q, k, v, pooled_k, pooled_v, pooled_dtype, selected_ids,
                                    selected_counts, pruned_ids, pruned_counts, dtype, q_heads,
                                    kv_heads, padded_q_len, padded_k_len, head_dim, offset,
                                    query_length, key_length, scale, block_k, tile_q,
                                    mean_correction, nullptr, out_multicast, head_offset,
                                    heads_total, workspace, workspace_bytes, stream);
}

int fpv2_sparse_attention_paged(
    const void* q, const void* k_pages, const void* v_pages, const int32_t* block_table,
    int32_t table_len, int32_t num_pages, int32_t page_size, const void* pooled_k,
    const void* pooled_v, int pooled_dtype, const int32_t* selected_ids,
    const int32_t* selected_counts, const int32_t* pruned_ids, const int32_t* pruned_counts,
    int dtype, int32_t q_heads, int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len,
    int32_t head_dim, int32_t offset, int32_t query_length, int32_t key_length, float scale,
    int32_t block_k, int32_t tile_q, int32_t mean_correction, void* out, void* workspace,
    int64_t workspace_bytes, void* stream) {
  const fpv2::PagedKV paged{block_table, table_len, num_pages, page_size};
  return fpv2::run_sparse_attention(q, k_pages, v_pages, pooled_k, pooled_v, pooled_dtype,
                                    selected_ids, selected_counts, pruned_ids, pruned_counts, dtype,
                                    q_heads, kv_heads, padded_q_len, padded_k_len, head_dim, offset,
                                    query_length, key_length, scale, block_k, tile_q,
                                    mean_correction, out, nullptr, 0, 0, workspace, workspace_bytes,
                                    stream, &paged);
}

int fpv2_pool_pages(const void* pages, const int32_t* block_table, int32_t table_len,
                    int32_t num_pages, int32_t page_size, int32_t kv_heads, int32_t head_dim,
                    int32_t length, int32_t block_size, int dtype, void* out, int out_dtype,
                    void* stream) {
  using namespace fpv2;
  if (dtype != DT_F16 && dtype != DT_BF16)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "page pools must be float16 or bfloat16");
  if (out_dtype != DT_F16 && out_dtype != DT_BF16 && out_dtype != DT_F32)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "unsupported output dtype");
  if (!pages || !block_table || !out) return fail(FPV2_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (kv_heads <= 0 || head_dim <= 0 || head_dim % 8 || page_size <= 0 || num_pages <= 0 ||
      table_len <= 0 || block_size <= 0)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "invalid page pool geometry");
  if (length <= 0 || length % block_size)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "sequence length must be divisible by block size");
  if ((long long)table_len * page_size < length)
    return fail(FPV2_ERR_INVALID_ARGUMENT, "block table does not cover the sequence");
  PagedPoolArgs a{pages, block_table, table_len, num_pages, page_size, kv_heads, head_dim, length,
                  block_size, out};
  cudaError_t e = launch_pool_pages(a, dtype, out_dtype, reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pool_pages launch");
  return FPV2_OK;
}

int fpv2_fast_path_mask(int dtype, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                        int32_t block_k, int32_t tile_q, int32_t num_blocks) {
  if (kv_heads <= 0 || q_heads % kv_heads) return 0;
  SelectGeom g{};
  g.Hq = q_heads;
  g.Hkv = kv_heads;
  g.G = q_heads / kv_heads;
  g.D = head_dim;
  g.Nb = num_blocks;
  g.block_k = block_k;
  g.tile_q = tile_q;
  g.scale = 1.f;   // any positive softmax scale
  AttnArgs a{};
  a.dt = dtype;
  a.pooled_dt = dtype;
  a.D = head_dim;
  a.G = g.G;
  a.block_k = block_k;
  a.tile_q = tile_q;
  a.Nb = num_blocks;
  a.scale_log2 = 1.f;   // any positive softmax scale
  int m = 0;
  if (select_tc_supported(g, dtype)) m |= 1;
  if (attn_tc_supported(a) || attn_wide_supported(a)) m |= 2;
  if (attn_pair_supported(a)) m |= 4;
  return m;
}

int fpv2_selftest_wait_timeout(double budget_ms, void* stream) {
  DeviceInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != FPV2_OK) return rc;
  if (!(budget_ms > 0.0)) return fail(FPV2_ERR_INVALID_ARGUMENT, "budget must be positive");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  e = cudaMemsetAsync(d->status, 0, sizeof(int), s);
  if (e != cudaSuccess) return cuda_fail(e, "clear status");
  TcLaunch L = tc_launch(*d);
  L.budget = (long long)(budget_ms * (d->clock_khz > 0 ? d->clock_khz : 2.0e6));
  e = launch_wait_selftest(L, s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest launch");
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "selftest sync");
  int v = 0;
  e = cudaMemcpy(&v, d->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "read status");
  e = cudaMemset(d->status, 0, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "clear status");
  if (v & STATUS_TIMEOUT)
    return fail(FPV2_ERR_DEVICE_TIMEOUT, "bounded wait expired after %.3f ms (as designed)",
                budget_ms);
  return FPV2_OK;
}

}  // extern "C"
