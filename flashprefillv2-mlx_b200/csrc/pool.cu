// Block mean pooling: x [heads, length, D] -> out [heads, length / bs, D].
//
// Definition (shared with the CPU oracle): the exact mean of the block -- a
// float64 sum of the inputs divided by bs -- rounded to float32 and then to
// the output dtype with round-to-nearest-even. A float64 sum of a block of
// 16-bit floats is exact whenever the block's nonzero magnitudes span fewer
// than ~28 binades, so the result does not depend on the summation order and
// is reproduced bit for bit.
//
// HBM-streaming kernel: one CTA per (tensor, head, block); 16-byte vector
// loads of 8 consecutive features per thread, rows spread over the CTA.
#include "common.cuh"
#include "kernels.h"

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

template <int DT_IN, int DT_OUT>
cudaError_t launch_pool_t(const PoolArgs& a, int ntensors, cudaStream_t stream) {
  const int64_t nblocks = a.heads * (a.length / a.bs);
  if (nblocks == 0) return cudaSuccess;
  dim3 grid((unsigned)nblocks, (unsigned)ntensors);
  constexpr int kPerVec = 16 / (int)sizeof(typename Elem<DT_IN>::T);
  bool vec = (a.D % kPerVec == 0) && (kPoolThreads % (a.D / kPerVec) == 0);
  for (int t = 0; t < ntensors && vec; ++t)
    vec = (reinterpret_cast<uintptr_t>(a.x[t]) % 16 == 0);
  if (vec) {
    const int rows_in_flight = kPoolThreads / (a.D / kPerVec);
    const size_t smem = sizeof(double) * (size_t)rows_in_flight * a.D;
    if (smem > 48 * 1024) vec = false;
    else {
      pool_vec_kernel<DT_IN, DT_OUT><<<grid, kPoolThreads, smem, stream>>>(a);
      return cudaGetLastError();
    }
  }
  pool_scalar_kernel<DT_IN, DT_OUT><<<grid, kPoolThreads, 0, stream>>>(a);
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

}  // namespace fpv2
