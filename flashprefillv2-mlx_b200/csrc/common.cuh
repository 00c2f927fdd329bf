// Shared device helpers for the FPV2 sm_100a kernels: element conversion,
// mbarriers with bounded waits, TMA (cp.async.bulk.tensor) and tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads and stores).
//
// Every wait in these kernels is bounded: a wait that exceeds its clock64
// budget sets a bit in the device status word, raises the CTA's abort flag
// and returns false, so the kernel unwinds instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fpv2 {

enum : int { DT_F16 = 0, DT_BF16 = 1, DT_F32 = 2 };

// Status bits written by kernels (fpv2_device_status).
enum : int {
  STATUS_TIMEOUT = 1,      // a bounded wait expired
  STATUS_TMEM_ALLOC = 2,   // TMEM allocation returned an unusable address
  STATUS_BAD_SPLIT = 4,    // a split-queue entry or partial slot failed its bounds check
  STATUS_BAD_LIST = 8,     // (FPV2_DEBUG_BOUNDS builds) a list entry or count was out of range
};

#ifndef FPV2_DEBUG_BOUNDS
#define FPV2_DEBUG_BOUNDS 0
#endif

// A block-list entry, count or page index clamped into [lo, hi], as the
// reference clips its lists (fpv2/kernel.py:555-558). A build with
// FPV2_DEBUG_BOUNDS=1 also reports every value that needed the clamp in the
// status word (STATUS_BAD_LIST) instead of trapping.
__device__ __forceinline__ int clamp_entry(int v, int lo, int hi, int* status) {
#if FPV2_DEBUG_BOUNDS
  if ((v < lo || v > hi) && status != nullptr) atomicOr(status, STATUS_BAD_LIST);
#else
  (void)status;
#endif
  return min(max(v, lo), hi);
}

constexpr float kFiniteMin = -3.402823466e+38f;  // Metal's Limits<float>::finite_min
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// element access
// ---------------------------------------------------------------------------

template <int DT> struct Elem;
template <> struct Elem<DT_F16> {
  using T = __half;
  static __device__ __forceinline__ float to_f(T x) { return __half2float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<DT_BF16> {
  using T = __nv_bfloat16;
  static __device__ __forceinline__ float to_f(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ T from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<DT_F32> {
  using T = float;
  static __device__ __forceinline__ float to_f(T x) { return x; }
  static __device__ __forceinline__ T from_f(float x) { return x; }
};

__device__ __forceinline__ float load_as_float(const void* p, int dt, int64_t i) {
  if (dt == DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// Two floats -> packed pair of 16-bit values, `lo` in the low half.
template <int DT> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<DT_BF16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <> __device__ __forceinline__ uint32_t pack2<DT_F16>(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
template <int DT> __device__ __forceinline__ float2 unpack2(uint32_t v);
template <> __device__ __forceinline__ float2 unpack2<DT_BF16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
template <> __device__ __forceinline__ float2 unpack2<DT_F16>(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2*>(&v);
  return __half22float2(h);
}

// Two-term split of float32 values into 16-bit pairs: the high part is
// round(x), the low part round(x - round(x)). Their sum carries about 16 (bf16)
// or 22 (fp16) significant bits, so a product accumulated over both parts in
// fp32 matches the float32 product to within float32 rounding.
template <int DT> __device__ __forceinline__ uint32_t pack2_split(float lo, float hi, bool low_part) {
  const uint32_t h = pack2<DT>(lo, hi);
  if (!low_part) return h;
  const float2 r = unpack2<DT>(h);
  return pack2<DT>(lo - r.x, hi - r.y);
}

// Packing of softmax probabilities p in [0, 2^16] for the P.V MMA. For bf16 the
// conversion is done on the integer units (round half up on the 16 dropped
// bits, then a byte permute), which keeps it off the pipe that evaluates ex2;
// it differs from round-to-nearest-even only on exact ties.
template <int DT> __device__ __forceinline__ uint32_t pack_p(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack_p<DT_BF16>(float lo, float hi) {
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <> __device__ __forceinline__ uint32_t pack_p<DT_F16>(float lo, float hi) {
  return pack2<DT_F16>(lo, hi);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100): one instruction does the work of two lanes.
__device__ __forceinline__ float2 fma_f32x2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add_f32x2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// max of three (sm_100 three-input max.f32)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for a pair, x <= 16, on the FMA and integer pipes instead of the MUFU:
// n = rint(x) through the 1.5 * 2^23 rounding constant, f = x - n in
// [-0.5, 0.5], 2^f by the minimax quartic for relative error on that
// interval (Remez exchange, levelled error 2.6e-6; tests/exp2_poly_fit.py
// reproduces the coefficients, and the float32 evaluation is checked below
// 2.7e-6 over the whole input range), and n added to the exponent field.
// Inputs below -126 are clamped (the result is then below 2^-125).
__device__ __forceinline__ float2 exp2_poly_x2(float2 x) {
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = add_f32x2(x, make_float2(12582912.f, 12582912.f));
  const float2 n = add_f32x2(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = fma_f32x2(n, make_float2(-1.f, -1.f), x);
  float2 p = fma_f32x2(make_float2(0.009570052f, 0.009570052f), f,
                       make_float2(0.055917736f, 0.055917736f));
  p = fma_f32x2(p, f, make_float2(0.24024744f, 0.24024744f));
  p = fma_f32x2(p, f, make_float2(0.69312185f, 0.69312185f));
  p = fma_f32x2(p, f, make_float2(0.99999928f, 0.99999928f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

// ---------------------------------------------------------------------------
// shared memory addressing
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

// Bounded wait context: the status word in global memory, the CTA abort flag
// in shared memory and the clock64 budget of one wait.
struct WaitCtx {
  int* status;
  volatile int* abort_flag;
  long long budget;
};

// Wait for the phase of `bar` with parity `parity` to complete. Returns false
// (after flagging) when the budget runs out or another role aborted.
// Drains of in-flight copies/MMAs pass honor_abort = false: they keep
// waiting (within the budget) even after another role aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w,
                                          bool honor_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (honor_abort && *w.abort_flag) return false;
    if (clock64() - t0 > w.budget) {
      atomicOr(w.status, STATUS_TIMEOUT);
      *w.abort_flag = 1;
      __threadfence_block();
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (tensor maps are __grid_constant__ kernel parameters)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Shared -> global tensor store (bulk-group completion).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the committed bulk stores have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until the committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 16-byte store to an NVLink multicast address: the switch writes it into the
// same offset of every GPU bound to the multicast object.
__device__ __forceinline__ void multimem_st16(void* gaddr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gaddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM, UMMA, loads/stores
// ---------------------------------------------------------------------------

// Allocate `ncols` TMEM columns (warp-collective); the address lands in *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a tile written by TMA with 128-byte
// swizzling: rows of 128 bytes, 8-row (1024-byte) swizzle atoms.
//   lbo/sbo are byte offsets (multiples of 16): K-major operands use
//   sbo = 1024 (next 8-row group) and an unused lbo of 16; MN-major operands
//   use lbo = distance between 64-element column groups and sbo = 1024.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;   // descriptor version for sm_100
  d |= (uint64_t)2 << 61;   // SWIZZLE_128B
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16 with fp32 accumulation.
//   ab_fmt: 0 = f16, 1 = bf16; a_mn/b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int ab_fmt, int M, int N, int a_mn, int b_mn) {
  return (1u << 4)                      // D format f32
         | ((uint32_t)ab_fmt << 7)      // A format
         | ((uint32_t)ab_fmt << 10)     // B format
         | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Orders later uses of `r` after a preceding tcgen05.wait::ld.
__device__ __forceinline__ void reg_fence(uint32_t (&r)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Named barrier for a subset of warps.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// Kernel launch record shared with the C-ABI layer (defined in capi.cu).
struct DeviceCtx {
  int* status;       // device status word of the current device
  long long budget;  // clock64 cycles per bounded wait
  int num_sms;
};

}  // namespace fpv2
