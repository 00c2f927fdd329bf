// Exact fp16 copy of bf16 V for the P.V product of the attention kernels.
//
// A tcgen05 MMA of kind::f16 takes A and B of one type, so P can only be held
// at fp16 precision (11 significant bits, against bf16's 8) if V is fp16 too.
// bf16 -> fp16 is exact for |v| in [2^-14, 65504]; smaller magnitudes lose at
// most 2^-25 in absolute terms, far below the output tolerance. Larger ones
// would overflow, so each KV head is scaled by 2^-e with e >= 0 the smallest
// exponent that brings its maximum magnitude within range (e = 0 for any
// ordinary activations); the attention epilogue multiplies the output by 2^e.
//
// Two launches: v_to_f16_kernel converts at e = 0 and records each head's
// maximum magnitude; v_rescale_kernel returns at once for heads within range
// and otherwise redoes the head with its exponent.
#include <algorithm>

#include "../../include/fpv2_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace fpv2 {
namespace {

constexpr int kConvThreads = 256;
constexpr float kF16Max = 65504.f;

// 16 bytes (8 values) of row `row`, column `col` of KV head h.
__device__ __forceinline__ const uint4* v_src(const VConvArgs& a, int h, long long row, int col) {
  const __nv_bfloat16* base = reinterpret_cast<const __nv_bfloat16*>(a.v);
  if (a.table == nullptr)
    return reinterpret_cast<const uint4*>(base + ((long long)h * a.L + row) * a.D + col);
  const int slot = (int)min(row / a.page_size, (long long)a.table_len - 1);
  const int page = min(max(a.table[slot], 0), a.num_pages - 1);
  const long long r = row % a.page_size;
  return reinterpret_cast<const uint4*>(base + (((long long)page * a.page_size + r) * a.Hkv + h) * a.D + col);
}

// 8 bf16 values times `scale` -> 8 fp16 values; `amax` tracks their magnitude.
__device__ __forceinline__ uint4 conv8(uint4 x, float scale, float& amax) {
  uint32_t w[4] = {x.x, x.y, x.z, x.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack2<DT_BF16>(w[i]);
    amax = max3f(amax, fabsf(f.x), fabsf(f.y));
    o[i] = pack2<DT_F16>(f.x * scale, f.y * scale);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ void convert_head(const VConvArgs& a, int h, float scale, float& amax) {
  const int vec_row = a.D / 8;
  const long long nvec = (long long)a.L * vec_row;
  uint4* dst = reinterpret_cast<uint4*>(a.v16) + (long long)h * nvec;
  const long long stride = (long long)gridDim.x * kConvThreads;
  long long i = (long long)blockIdx.x * kConvThreads + threadIdx.x;
  // four independent 16-byte loads in flight per thread before converting them
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    uint4 x[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long j = i + u * stride;
      x[u] = __ldg(v_src(a, h, j / vec_row, (int)(j % vec_row) * 8));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) dst[i + u * stride] = conv8(x[u], scale, amax);
  }
  for (; i < nvec; i += stride) dst[i] = conv8(__ldg(v_src(a, h, i / vec_row, (int)(i % vec_row) * 8)), scale, amax);
  if (a.pv != nullptr && blockIdx.x == 0) {   // pooled V: means of V, so within the same range
    const long long npv = (long long)a.Nb * vec_row;
    const uint4* src = reinterpret_cast<const uint4*>(a.pv) + (long long)h * npv;
    uint4* pdst = reinterpret_cast<uint4*>(a.pv16) + (long long)h * npv;
    float unused = 0.f;
    for (long long i = threadIdx.x; i < npv; i += kConvThreads) pdst[i] = conv8(__ldg(src + i), scale, unused);
  }
}

__global__ void __launch_bounds__(kConvThreads) v_to_f16_kernel(VConvArgs a) {
  const int h = blockIdx.y;
  float amax = 0.f;
  convert_head(a, h, 1.f, amax);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) atomicMax(a.absmax + h, __float_as_uint(amax));   // amax >= 0
  if (blockIdx.x == 0 && threadIdx.x == 0) a.v_exp[h] = 0;
}

__global__ void __launch_bounds__(kConvThreads) v_rescale_kernel(VConvArgs a) {
  const int h = blockIdx.y;
  const float amax = __uint_as_float(a.absmax[h]);
  // the exact copy stands (an infinite value stays infinite, as in the bf16 product)
  if (!(amax > kF16Max) || isinf(amax)) return;
  int e = 0;
  while (ldexpf(amax, -e) > kF16Max && e < 200) ++e;
  float unused = 0.f;
  convert_head(a, h, ldexpf(1.f, -e), unused);
  if (blockIdx.x == 0 && threadIdx.x == 0) a.v_exp[h] = e;
}

size_t up256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

size_t v_conv_bytes(int Hkv, int L, int D, int Nb) {
  return up256((size_t)Hkv * L * D * 2) + up256((size_t)Hkv * Nb * D * 2) + up256((size_t)Hkv * 8);
}

cudaError_t launch_v_to_f16(const VConvArgs& a, cudaStream_t stream) {
  if (a.D % 8 != 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaMemsetAsync(a.absmax, 0, sizeof(unsigned) * a.Hkv, stream);
  if (e != cudaSuccess) return e;
  const long long nvec = (long long)a.L * (a.D / 8);
  const int bx = (int)std::min<long long>((nvec + kConvThreads * 8 - 1) / (kConvThreads * 8), 1024);
  const dim3 grid(std::max(bx, 1), a.Hkv);
  v_to_f16_kernel<<<grid, kConvThreads, 0, stream>>>(a);
  v_rescale_kernel<<<grid, kConvThreads, 0, stream>>>(a);
  count_launch();
  count_launch();
  return cudaGetLastError();
}

}  // namespace fpv2
