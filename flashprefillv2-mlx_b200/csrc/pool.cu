// Block mean pooling: x [heads, length, D] -> out [heads, length / bs, D].
//
// Definition (shared with the CPU oracle): the exact mean of the block -- a
// float64 sum of the inputs divided by bs -- rounded to float32 and then to
// the output dtype with round-to-nearest-even. A float64 sum of a block of
// 16-bit floats is exact whenever the block's nonzero magnitudes span fewer
// than ~28 binades, so the result does not depend on the summation order and
// is reproduced bit for bit.
//
// Streaming kernels. For 16-bit inputs whose blocks are at most 32 KB (the
// configurations the hook runs), persistent CTAs stream whole blocks (one
// contiguous bs x D run each) through a 3-stage shared-memory ring with
// cp.async, so the loads of the next blocks are in flight while the current
// block is summed; other shapes take one CTA per (tensor, head, block) with
// 16-byte vector loads of 8 consecutive features per thread.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace fpv2 {

namespace {

constexpr int kPoolThreads = 256;

template <int DT_IN, int DT_OUT>
__global__ void __launch_bounds__(kPoolThreads)
    pool_vec_kernel(PoolArgs a) {
  using Tin = typename Elem<DT_IN>::T;
  using Tout = typename Elem<DT_OUT>::T;
  constexpr int kPerVec = 16 / sizeof(Tin);        // elements per 16-byte load
  const bool second = blockIdx.y != 0;
  const Tin* __restrict__ x = reinterpret_cast<const Tin*>(second ? a.x[1] : a.x[0]);
  Tout* __restrict__ out = reinterpret_cast<Tout*>(second ? a.out[1] : a.out[0]);
  const int64_t nblk = a.length / a.bs;
  const int64_t hb = blockIdx.x;                   // head * nblk + block
  const int vec_per_row = a.D / kPerVec;
  const int rows_in_flight = kPoolThreads / vec_per_row;
  const int tid = threadIdx.x;
  const int vcol = tid % vec_per_row;
  const int rsub = tid / vec_per_row;
  const int64_t head = hb / nblk;
  const int64_t blk = hb % nblk;
  const Tin* base = x + (head * a.length + blk * a.bs) * a.D + vcol * kPerVec;

  double acc[kPerVec];
#pragma unroll
  for (int i = 0; i < kPerVec; ++i) acc[i] = 0.0;
  if (rsub < rows_in_flight) {
    // Issue 8 independent 16-byte loads before accumulating (memory-level parallelism).
    constexpr int kBatch = 8;
    for (int r0 = rsub; r0 < a.bs; r0 += kBatch * rows_in_flight) {
      uint4 raw[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int r = r0 + u * rows_in_flight;
        raw[u] = r < a.bs ? __ldg(reinterpret_cast<const uint4*>(base + (int64_t)r * a.D))
                          : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const Tin* e = reinterpret_cast<const Tin*>(&raw[u]);
#pragma unroll
        for (int i = 0; i < kPerVec; ++i) acc[i] += (double)Elem<DT_IN>::to_f(e[i]);
      }
    }
  }
  // Reduce the row groups: [rows_in_flight][D] partial sums in shared memory.
  extern __shared__ double red[];
  if (rsub < rows_in_flight) {
#pragma unroll
    for (int i = 0; i < kPerVec; ++i) red[rsub * a.D + vcol * kPerVec + i] = acc[i];
  }
  __syncthreads();
  for (int c = tid; c < a.D; c += kPoolThreads) {
    double s = 0.0;
    for (int r = 0; r < rows_in_flight; ++r) s += red[r * a.D + c];
    const float m = (float)(s / (double)a.bs);
    out[hb * a.D + c] = Elem<DT_OUT>::from_f(m);
  }
}

template <int DT_IN, int DT_OUT>
__global__ void __launch_bounds__(kPoolThreads)
    pool_scalar_kernel(PoolArgs a) {
  using Tin = typename Elem<DT_IN>::T;
  using Tout = typename Elem<DT_OUT>::T;
  const bool second = blockIdx.y != 0;
  const Tin* __restrict__ x = reinterpret_cast<const Tin*>(second ? a.x[1] : a.x[0]);
  Tout* __restrict__ out = reinterpret_cast<Tout*>(second ? a.out[1] : a.out[0]);
  const int64_t nblk = a.length / a.bs;
  const int64_t hb = blockIdx.x;
  const int64_t head = hb / nblk;
  const int64_t blk = hb % nblk;
  const Tin* base = x + (head * a.length + blk * a.bs) * a.D;
  for (int c = threadIdx.x; c < a.D; c += kPoolThreads) {
    double s = 0.0;
    for (int r = 0; r < a.bs; ++r) s += (double)Elem<DT_IN>::to_f(base[(int64_t)r * a.D + c]);
    out[hb * a.D + c] = Elem<DT_OUT>::from_f((float)(s / (double)a.bs));
  }
}


// ---- pipelined kernel ------------------------------------------------------
constexpr int kPipeThreads = 256;
constexpr int kPipeStages = 3;
constexpr int kPipeMaxUnitBytes = 32 * 1024;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One unit = one (tensor, head, block): `bs` consecutive rows of D features,
// contiguous in memory. Unit u of ntensors * heads * nblk; tensor-major.
template <int DT_IN, int DT_OUT>
__global__ void __launch_bounds__(kPipeThreads)
    pool_pipe_kernel(PoolArgs a, int ntensors) {
  using Tout = typename Elem<DT_OUT>::T;
  constexpr int kPerVec = 8;                               // 16-bit features per 16 bytes
  extern __shared__ __align__(16) uint8_t pool_smem[];
  const int cpr = a.D / kPerVec;                           // 16-byte chunks per row
  const int unit_chunks = (int)a.bs * cpr;                 // multiple of kPipeThreads
  const int unit_bytes = unit_chunks * 16;
  const uint32_t ring = smem_u32(pool_smem);
  double* red = reinterpret_cast<double*>(pool_smem + kPipeStages * unit_bytes);
  const int64_t nblk = a.length / a.bs;
  const int64_t per_tensor = a.heads * nblk;
  const int64_t units = per_tensor * ntensors;
  const int tid = threadIdx.x;
  const uint8_t* const x0 = reinterpret_cast<const uint8_t*>(a.x[0]);
  const uint8_t* const x1 = reinterpret_cast<const uint8_t*>(a.x[1]);
  auto issue = [=](int64_t u, int stage) {
    if (u < units) {
      const int t = (int)(u / per_tensor);
      const int64_t hb = u % per_tensor;                   // head * nblk + block, rows contiguous
      const uint8_t* src = (t == 0 ? x0 : x1) + hb * (int64_t)unit_bytes;
      const uint32_t dst = ring + stage * unit_bytes;
      for (int q = tid; q < unit_chunks; q += kPipeThreads) cp_async16(dst + q * 16, src + q * 16);
    }
    cp_async_commit();   // one group per unit slot, empty past the end
  };
  int64_t u = blockIdx.x;
#pragma unroll
  for (int s = 0; s < kPipeStages - 1; ++s) issue(u + (int64_t)s * gridDim.x, s);
  const int c = tid % cpr;                                 // this thread's 8 features
  const int rstep = kPipeThreads / cpr;
  for (int i = 0; u < units; ++i, u += gridDim.x) {
    issue(u + (int64_t)(kPipeStages - 1) * gridDim.x, (i + kPipeStages - 1) % kPipeStages);
    cp_async_wait<kPipeStages - 1>();                      // this unit's copies (own) landed
    __syncthreads();                                       // ... and everyone else's
    const uint8_t* st = pool_smem + (i % kPipeStages) * unit_bytes;
    double acc[kPerVec];
#pragma unroll
    for (int e = 0; e < kPerVec; ++e) acc[e] = 0.0;
    for (int r = tid / cpr; r < a.bs; r += rstep) {
      const uint4 raw = *reinterpret_cast<const uint4*>(st + (r * cpr + c) * 16);
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack2<DT_IN>(w[e]);
        acc[2 * e] += (double)f.x;
        acc[2 * e + 1] += (double)f.y;
      }
    }
    const int j = tid / cpr;
#pragma unroll
    for (int e = 0; e < kPerVec; ++e) red[j * a.D + c * kPerVec + e] = acc[e];
    __syncthreads();
    for (int col = tid; col < a.D; col += kPipeThreads) {
      double sum = 0.0;
      for (int jj = 0; jj < rstep; ++jj) sum += red[jj * a.D + col];
      const float m = (float)(sum / (double)a.bs);
      const int t = (int)(u / per_tensor);
      Tout* out = reinterpret_cast<Tout*>(t == 0 ? a.out[0] : a.out[1]);
      out[(u % per_tensor) * a.D + col] = Elem<DT_OUT>::from_f(m);
    }
    __syncthreads();                                       // ring stage and red reusable
  }
  cp_async_wait<0>();
}

template <int DT_IN, int DT_OUT>
cudaError_t launch_pool_t(const PoolArgs& a, int ntensors, cudaStream_t stream) {
  const int64_t nblocks = a.heads * (a.length / a.bs);
  if (nblocks == 0) return cudaSuccess;
  dim3 grid((unsigned)nblocks, (unsigned)ntensors);
  constexpr int kPerVec = 16 / (int)sizeof(typename Elem<DT_IN>::T);
  if constexpr (kPerVec == 8) {
   if (a.D % 8 == 0 && kPipeThreads % (a.D / 8) == 0 &&
      (a.bs * (a.D / 8)) % kPipeThreads == 0 && a.bs * a.D * 2 <= kPipeMaxUnitBytes) {
    bool aligned = true;
    for (int t = 0; t < ntensors; ++t) aligned &= reinterpret_cast<uintptr_t>(a.x[t]) % 16 == 0;
    if (aligned) {
      int dev = 0, sms = 0;
      cudaError_t e = cudaGetDevice(&dev);
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return e;
      const int unit_bytes = (int)(a.bs * a.D * 2);
      const size_t smem = (size_t)kPipeStages * unit_bytes +
                          sizeof(double) * (size_t)(kPipeThreads / (a.D / 8)) * a.D;
      e = cudaFuncSetAttribute(pool_pipe_kernel<DT_IN, DT_OUT>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      const int64_t units = nblocks * ntensors;
      const int g = (int)std::min<int64_t>(units, 2 * (int64_t)sms);   // two CTAs per SM
      pool_pipe_kernel<DT_IN, DT_OUT><<<g, kPipeThreads, smem, stream>>>(a, ntensors);
      count_launch();
      return cudaGetLastError();
    }
   }
  }
  bool vec = (a.D % kPerVec == 0) && (kPoolThreads % (a.D / kPerVec) == 0);
  for (int t = 0; t < ntensors && vec; ++t)
    vec = (reinterpret_cast<uintptr_t>(a.x[t]) % 16 == 0);
  if (vec) {
    const int rows_in_flight = kPoolThreads / (a.D / kPerVec);
    const size_t smem = sizeof(double) * (size_t)rows_in_flight * a.D;
    if (smem > 48 * 1024) vec = false;
    else {
      pool_vec_kernel<DT_IN, DT_OUT><<<grid, kPoolThreads, smem, stream>>>(a);
      count_launch();
      return cudaGetLastError();
    }
  }
  pool_scalar_kernel<DT_IN, DT_OUT><<<grid, kPoolThreads, 0, stream>>>(a);
  count_launch();
  return cudaGetLastError();
}


// ---- paged sequences ---------------------------------------------------------
// One CTA per (head, block); rows of the block are looked up in the block table
// (row p of the sequence = row p % page_size of page table[p / page_size]).
template <int DT_IN, int DT_OUT>
__global__ void __launch_bounds__(kPoolThreads)
    pool_pages_kernel(PagedPoolArgs a) {
  using Tout = typename Elem<DT_OUT>::T;
  const int nblk = a.length / a.bs;
  const int head = blockIdx.x / nblk;
  const int blk = blockIdx.x % nblk;
  const int cpr = a.D / 8;                          // 16-byte chunks per row
  const int rows_in_flight = kPoolThreads / cpr;
  const int tid = threadIdx.x;
  const int c = tid % cpr, rsub = tid / cpr;
  double acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.0;
  if (rsub < rows_in_flight) {
    for (int r = rsub; r < a.bs; r += rows_in_flight) {
      const int pos = blk * a.bs + r;
      const int page = min(max(a.table[pos / a.page_size], 0), a.num_pages - 1);
      const long long row = ((long long)page * a.page_size + pos % a.page_size) * a.heads + head;
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(
          reinterpret_cast<const uint8_t*>(a.pages) + (row * a.D + c * 8) * 2));
      const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack2<DT_IN>(w[e]);
        acc[2 * e] += (double)f.x;
        acc[2 * e + 1] += (double)f.y;
      }
    }
  }
  extern __shared__ double pred[];
  if (rsub < rows_in_flight) {
#pragma unroll
    for (int e = 0; e < 8; ++e) pred[rsub * a.D + c * 8 + e] = acc[e];
  }
  __syncthreads();
  for (int col = tid; col < a.D; col += kPoolThreads) {
    double sum = 0.0;
    for (int j = 0; j < rows_in_flight; ++j) sum += pred[j * a.D + col];
    const float m = (float)(sum / (double)a.bs);
    reinterpret_cast<Tout*>(a.out)[((long long)head * nblk + blk) * a.D + col] = Elem<DT_OUT>::from_f(m);
  }
}

template <int DT_IN, int DT_OUT>
cudaError_t launch_pool_pages_t(const PagedPoolArgs& a, cudaStream_t stream) {
  const int cpr = a.D / 8;
  if (cpr > kPoolThreads) return cudaErrorInvalidValue;   // threads past whole rows idle
  const int nblocks = a.heads * (a.length / a.bs);
  const size_t smem = sizeof(double) * (size_t)(kPoolThreads / cpr) * a.D;
  pool_pages_kernel<DT_IN, DT_OUT><<<nblocks, kPoolThreads, smem, stream>>>(a);
  count_launch();
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_pool(const PoolArgs& a, int ntensors, int dt_in, int dt_out,
                        cudaStream_t stream) {
#define FPV2_POOL_CASE(I, O) \
  if (dt_in == I && dt_out == O) return launch_pool_t<I, O>(a, ntensors, stream);
  FPV2_POOL_CASE(DT_BF16, DT_BF16)
  FPV2_POOL_CASE(DT_BF16, DT_F32)
  FPV2_POOL_CASE(DT_F16, DT_F16)
  FPV2_POOL_CASE(DT_F16, DT_F32)
  FPV2_POOL_CASE(DT_F32, DT_F32)
  FPV2_POOL_CASE(DT_F32, DT_BF16)
  FPV2_POOL_CASE(DT_F32, DT_F16)
  FPV2_POOL_CASE(DT_BF16, DT_F16)
  FPV2_POOL_CASE(DT_F16, DT_BF16)
#undef FPV2_POOL_CASE
  return cudaErrorInvalidValue;
}

cudaError_t launch_pool_pages(const PagedPoolArgs& a, int dt_in, int dt_out, cudaStream_t stream) {
  if (a.heads <= 0 || a.length / a.bs == 0) return cudaSuccess;
#define FPV2_PAGES_CASE(I, O) \
  if (dt_in == I && dt_out == O) return launch_pool_pages_t<I, O>(a, stream);
  FPV2_PAGES_CASE(DT_BF16, DT_BF16)
  FPV2_PAGES_CASE(DT_BF16, DT_F32)
  FPV2_PAGES_CASE(DT_F16, DT_F16)
  FPV2_PAGES_CASE(DT_F16, DT_F32)
#undef FPV2_PAGES_CASE
  return cudaErrorInvalidValue;
}

}  // namespace fpv2
