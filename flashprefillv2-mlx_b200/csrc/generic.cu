// Generic CUDA-core kernels: selection for any dtype/head_dim/tile shape,
// raw scores, mask compaction and block-sparse attention for shapes the
// tcgen05 kernels do not cover (odd head dims, small tiles, block_k < 128).
//
// Selection follows fpv2/selection.py:144-195 literally: two passes per
// (KV head, tile) -- the tile max over fully visible blocks and visible rows,
// then per-block sums of exp(score - max) -- with float32 scores.
// Attention follows the Metal kernel fpv2/kernel.py:187-414: online softmax
// in base 2, masked logits at finite_min, then the pooled correction with the
// log2(block_k) shift.
#include "common.cuh"
#include "kernels.h"

namespace fpv2 {

namespace {

constexpr int kSelThreads = 256;
constexpr int kSelRows = 16;   // query rows staged per pass

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide max over kSelThreads threads (uses red[0..8]).
__device__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kSelThreads / 32; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

// One CTA per (kv head, tile).  Dynamic smem: q rows [kSelRows][D] floats,
// then energies[Nb] floats.
__global__ void __launch_bounds__(kSelThreads)
    select_generic_kernel(SelectGeom g, const void* __restrict__ q, int q_dt,
                          const void* __restrict__ pk, int pk_dt, uint8_t* __restrict__ mask,
                          SelectLists lists) {
  extern __shared__ float sm[];
  float* qs = sm;
  float* energy = sm + kSelRows * g.D;
  uint8_t* fin = reinterpret_cast<uint8_t*>(energy + g.Nb);
  __shared__ float red[32];
  const int h = blockIdx.x / g.Nt;
  const int t = blockIdx.x % g.Nt;
  const int R = g.G * g.tile_q;
  const long long tile_first = (long long)g.offset + (long long)t * g.tile_q;
  const long long tile_last =
      min(tile_first + g.tile_q, (long long)g.offset + g.valid_lq) - 1;
  // Fully visible blocks: block_end <= tile_last + 1 (blocks are ascending).
  int n_full = 0;
  if (tile_last + 1 >= g.block_k) n_full = (int)min((long long)g.Nb, (tile_last + 1) / g.block_k);

  for (int b = threadIdx.x; b < g.Nb; b += kSelThreads) energy[b] = 0.f;

  float M = -INFINITY;
  for (int pass = 0; pass < 2 && n_full > 0; ++pass) {
    float local_max = -INFINITY;
    for (int r0 = 0; r0 < R; r0 += kSelRows) {
      const int nr = min(kSelRows, R - r0);
      __syncthreads();
      for (int i = threadIdx.x; i < nr * g.D; i += kSelThreads) {
        const int rr = r0 + i / g.D, d = i % g.D;
        const int gg = rr / g.tile_q, pos = rr % g.tile_q;
        const long long row = (long long)t * g.tile_q + pos;
        const long long qi = (((long long)(h * g.G + gg)) * g.Lq_pad + row) * g.D + d;
        qs[i] = load_as_float(q, q_dt, qi);
      }
      __syncthreads();
      for (int b = threadIdx.x; b < n_full; b += kSelThreads) {
        const long long kbase = ((long long)h * g.Nb + b) * g.D;
        float acc[kSelRows];
#pragma unroll
        for (int r = 0; r < kSelRows; ++r) acc[r] = 0.f;
        for (int d = 0; d < g.D; ++d) {
          const float kv = load_as_float(pk, pk_dt, kbase + d);
#pragma unroll
          for (int r = 0; r < kSelRows; ++r) acc[r] = fmaf(qs[r * g.D + d], kv, acc[r]);
        }
        float e = 0.f;
        for (int r = 0; r < nr; ++r) {
          const int rr = r0 + r;
          const long long row = (long long)t * g.tile_q + rr % g.tile_q;
          const bool ok = row < g.valid_lq && (long long)b * g.block_k <= g.offset + row;
          if (!ok) continue;
          const float s = acc[r] * g.scale;
          if (pass == 0) local_max = fmaxf(local_max, s);
          else e += expf(s - M);
        }
        if (pass == 1) energy[b] += e;
      }
    }
    if (pass == 0) M = block_max(local_max, red);
    if (M == -INFINITY) break;   // nothing visible: every energy stays 0
  }
  __syncthreads();
  float emax = 0.f;
  for (int b = threadIdx.x; b < g.Nb; b += kSelThreads) emax = fmaxf(emax, energy[b]);
  emax = block_max(emax, red);
  const float thr = g.alpha * emax;
  const bool dense_tail = t >= max(g.Nt - g.last_n, 0);
  const long long row_base = ((long long)h * g.Nt + t) * g.Nb;
  for (int b = threadIdx.x; b < g.Nb; b += kSelThreads) {
    const long long bs = (long long)b * g.block_k, be = bs + g.block_k;
    const bool sel = energy[b] >= thr;
    const bool forced = bs < g.sink || be > tile_first - g.window || dense_tail;
    const bool visible = bs <= tile_last;
    const uint8_t f = (uint8_t)((sel || forced) && visible);
    fin[b] = f;
    if (mask != nullptr) mask[row_base + b] = f;
  }
  if (lists.sel_ids == nullptr) return;
  __syncthreads();
  if (threadIdx.x < 32) {
    // Ballot compaction of this tile's mask (same order as compact_kernel).
    const int lane = threadIdx.x;
    const unsigned lt = (1u << lane) - 1u;
    int nsel = 0, npr = 0;
    for (int c = 0; c < g.Nb; c += 32) {
      const int b = c + lane;
      const bool sb = b < g.Nb && fin[b];
      const long long be = min((long long)(b + 1) * g.block_k, (long long)g.valid_lk);
      const bool pb = b < g.Nb && !sb && be <= tile_first;
      nsel += __popc(__ballot_sync(0xffffffffu, sb));
      npr += __popc(__ballot_sync(0xffffffffu, pb));
    }
    int sel_before = 0, pr_before = 0;
    for (int c = 0; c < g.Nb; c += 32) {
      const int b = c + lane;
      const bool sb = b < g.Nb && fin[b];
      const long long be = min((long long)(b + 1) * g.block_k, (long long)g.valid_lk);
      const bool pb = b < g.Nb && !sb && be <= tile_first;
      const unsigned bsel = __ballot_sync(0xffffffffu, sb);
      const unsigned bpr = __ballot_sync(0xffffffffu, pb);
      if (b < g.Nb) {
        const int rs = sel_before + __popc(bsel & lt);
        lists.sel_ids[row_base + (sb ? rs : nsel + (b - rs))] = b;
        const int rp = pr_before + __popc(bpr & lt);
        lists.pr_ids[row_base + (pb ? rp : npr + (b - rp))] = b;
      }
      sel_before += __popc(bsel);
      pr_before += __popc(bpr);
    }
    if (lane == 0) {
      lists.sel_counts[(long long)h * g.Nt + t] = nsel;
      lists.pr_counts[(long long)h * g.Nt + t] = npr;
    }
  }
}

__global__ void raw_scores_kernel(SelectGeom g, const void* __restrict__ q, int q_dt,
                                  const void* __restrict__ pk, int pk_dt, float* __restrict__ out) {
  extern __shared__ float qrow[];
  // blockIdx.x = row index over [Hq * Lq_pad]
  const long long hr = blockIdx.x;
  const int hq = (int)(hr / g.Lq_pad);
  const int h = hq / g.G;
  for (int d = threadIdx.x; d < g.D; d += blockDim.x) qrow[d] = load_as_float(q, q_dt, hr * g.D + d);
  __syncthreads();
  for (int b = threadIdx.x; b < g.Nb; b += blockDim.x) {
    const long long kbase = ((long long)h * g.Nb + b) * g.D;
    float acc = 0.f;
    for (int d = 0; d < g.D; ++d) acc = fmaf(qrow[d], load_as_float(pk, pk_dt, kbase + d), acc);
    out[hr * g.Nb + b] = acc * g.scale;
  }
}

// One warp per (kv head, tile) row of the mask.
__global__ void compact_kernel(const uint8_t* __restrict__ mask, int rows, int Nt, int Nb,
                               int block_k, int tile_q, int offset, int valid_lk,
                               int32_t* __restrict__ sel_ids, int32_t* __restrict__ sel_counts,
                               int32_t* __restrict__ pr_ids, int32_t* __restrict__ pr_counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int t = warp % Nt;
  const long long tile_first = (long long)offset + (long long)t * tile_q;
  const uint8_t* m = mask + (long long)warp * Nb;
  const unsigned lt = (1u << lane) - 1u;
  int nsel = 0, npr = 0;
  for (int c = 0; c < Nb; c += 32) {
    const int b = c + lane;
    const bool s = b < Nb && m[b];
    const long long be = min((long long)(b + 1) * block_k, (long long)valid_lk);
    const bool p = b < Nb && !s && be <= tile_first;
    nsel += __popc(__ballot_sync(0xffffffffu, s));
    npr += __popc(__ballot_sync(0xffffffffu, p));
  }
  int32_t* so = sel_ids + (long long)warp * Nb;
  int32_t* po = pr_ids + (long long)warp * Nb;
  int sel_before = 0, pr_before = 0;
  for (int c = 0; c < Nb; c += 32) {
    const int b = c + lane;
    const bool s = b < Nb && m[b];
    const long long be = min((long long)(b + 1) * block_k, (long long)valid_lk);
    const bool p = b < Nb && !s && be <= tile_first;
    const unsigned bs = __ballot_sync(0xffffffffu, s);
    const unsigned bp = __ballot_sync(0xffffffffu, p);
    if (b < Nb) {
      const int rs = sel_before + __popc(bs & lt);          // selected blocks before b
      so[s ? rs : nsel + (b - rs)] = b;
      const int rp = pr_before + __popc(bp & lt);
      po[p ? rp : npr + (b - rp)] = b;
    }
    sel_before += __popc(bs);
    pr_before += __popc(bp);
  }
  if (lane == 0) {
    sel_counts[warp] = nsel;
    pr_counts[warp] = npr;
  }
}

// ---- generic attention: one warp per query row -----------------------------
constexpr int kAttnWarps = 4;
constexpr int kMaxDPerLane = 8;   // head_dim <= 256

template <int DT>
__device__ __forceinline__ float round_dt(float x) {
  return Elem<DT>::to_f(Elem<DT>::from_f(x));
}

template <int DT>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_generic_kernel(AttnArgs a) {
  using T = typename Elem<DT>::T;
  extern __shared__ float qsm[];   // [kAttnWarps][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long grow = (long long)blockIdx.x * kAttnWarps + warp;   // over Hq * Lq_pad
  if (grow >= (long long)a.Hq * a.Lq_pad) return;
  const int hq = (int)(grow / a.Lq_pad);
  const int row = (int)(grow % a.Lq_pad);
  const int h = hq / a.G;
  const int t = row / a.tile_q;
  const T* q = reinterpret_cast<const T*>(a.q);
  const T* k = reinterpret_cast<const T*>(a.k);
  const T* v = reinterpret_cast<const T*>(a.v);
  float* qrow = qsm + warp * a.D;
  for (int d = lane; d < a.D; d += 32) qrow[d] = Elem<DT>::to_f(q[grow * a.D + d]);
  __syncwarp();
  const long long position = (long long)a.offset + row;
  const bool row_valid = row < a.valid_lq;
  // Last valid position of the tile: blocks starting beyond it are skipped
  // (fpv2/kernel.py:249-255).
  const long long abs_last =
      (long long)a.offset + min((long long)(t + 1) * a.tile_q, (long long)a.valid_lq) - 1;
  const long long list_row = ((long long)h * a.Nt + t) * a.Nb;
  float o[kMaxDPerLane];
#pragma unroll
  for (int i = 0; i < kMaxDPerLane; ++i) o[i] = 0.f;
  float m_run = kFiniteMin, l_run = 0.f;

  const int nsel = clamp_entry(a.sel_counts[(long long)h * a.Nt + t], 0, a.Nb, a.status);
  for (int i = 0; i < nsel; ++i) {
    const int blk = clamp_entry(a.sel_ids[list_row + i], 0, a.Nb - 1, a.status);
    const long long bstart = (long long)blk * a.block_k;
    if (bstart > abs_last) break;
    for (int k0 = 0; k0 < a.block_k; k0 += 32) {
      const long long kpos = bstart + k0 + lane;
      if (bstart + k0 > abs_last) break;
      const bool kin = k0 + lane < a.block_k;
      float s = kFiniteMin;
      if (kin) {
        float acc = 0.f;
        const T* kr = k + ((long long)h * a.Lk_pad + kpos) * a.D;
        for (int d = 0; d < a.D; ++d) acc = fmaf(qrow[d], Elem<DT>::to_f(kr[d]), acc);
        const bool ok = row_valid && kpos < a.valid_lk && kpos <= position;
        if (ok) s = acc * a.scale_log2;
      }
      const float m_new = fmaxf(m_run, warp_max(kin ? s : kFiniteMin));
      const float resc = ex2(m_run - m_new);
      const float p = kin ? ex2(s - m_new) : 0.f;
      l_run = l_run * resc + warp_sum(p);
#pragma unroll
      for (int i2 = 0; i2 < kMaxDPerLane; ++i2) o[i2] *= resc;
      const int nk = min(32, a.block_k - k0);
      for (int j = 0; j < nk; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const T* vr = v + ((long long)h * a.Lk_pad + bstart + k0 + j) * a.D;
#pragma unroll
        for (int i2 = 0; i2 < kMaxDPerLane; ++i2) {
          const int d = lane + 32 * i2;
          if (d < a.D) o[i2] = fmaf(pj, Elem<DT>::to_f(vr[d]), o[i2]);
        }
      }
      m_run = m_new;
    }
  }
  if (a.corr) {
    const int npr = clamp_entry(a.pr_counts[(long long)h * a.Nt + t], 0, a.Nb, a.status);
    for (int e0 = 0; e0 < npr; e0 += 32) {
      const int e = e0 + lane;
      const bool in = e < npr;
      const int blk = clamp_entry(a.pr_ids[list_row + (in ? e : e0)], 0, a.Nb - 1, a.status);
      float s = kFiniteMin;
      if (in) {
        float acc = 0.f;
        const long long kb = ((long long)h * a.Nb + blk) * a.D;
        for (int d = 0; d < a.D; ++d)
          acc = fmaf(qrow[d], round_dt<DT>(load_as_float(a.pk, a.pooled_dt, kb + d)), acc);
        s = acc * a.scale_log2 + a.corr_shift;
      }
      const float m_new = fmaxf(m_run, warp_max(s));
      const float resc = ex2(m_run - m_new);
      const float p = in ? ex2(s - m_new) : 0.f;
      l_run = l_run * resc + warp_sum(p);
#pragma unroll
      for (int i2 = 0; i2 < kMaxDPerLane; ++i2) o[i2] *= resc;
      const int ne = min(32, npr - e0);
      for (int j = 0; j < ne; ++j) {
        const float pj = __shfl_sync(0xffffffffu, p, j);
        const int bj = __shfl_sync(0xffffffffu, blk, j);
        const long long vb = ((long long)h * a.Nb + bj) * a.D;
#pragma unroll
        for (int i2 = 0; i2 < kMaxDPerLane; ++i2) {
          const int d = lane + 32 * i2;
          if (d < a.D) o[i2] = fmaf(pj, round_dt<DT>(load_as_float(a.pv, a.pooled_dt, vb + d)), o[i2]);
        }
      }
      m_run = m_new;
    }
  }
  T* out = reinterpret_cast<T*>(a.out);
  const float inv = 1.f / l_run;
#pragma unroll
  for (int i2 = 0; i2 < kMaxDPerLane; ++i2) {
    const int d = lane + 32 * i2;
    if (d < a.D) out[grow * a.D + d] = Elem<DT>::from_f(o[i2] * inv);
  }
}

}  // namespace

cudaError_t launch_select_generic(const SelectGeom& g, const void* q, int q_dt, const void* pk,
                                  int pk_dt, uint8_t* mask, const SelectLists& lists,
                                  cudaStream_t stream) {
  const size_t smem = sizeof(float) * ((size_t)kSelRows * g.D + g.Nb) + g.Nb + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(select_generic_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const long long nblk = (long long)g.Hkv * g.Nt;
  if (nblk == 0) return cudaSuccess;
  select_generic_kernel<<<(unsigned)nblk, kSelThreads, smem, stream>>>(g, q, q_dt, pk, pk_dt,
                                                                       mask, lists);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_raw_scores(const SelectGeom& g, const void* q, int q_dt, const void* pk,
                              int pk_dt, float* out, cudaStream_t stream) {
  const long long rows = (long long)g.Hq * g.Lq_pad;
  if (rows == 0) return cudaSuccess;
  raw_scores_kernel<<<(unsigned)rows, 128, sizeof(float) * g.D, stream>>>(g, q, q_dt, pk, pk_dt,
                                                                          out);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_compact(const uint8_t* mask, int Hkv, int Nt, int Nb, int block_k, int tile_q,
                           int offset, int valid_lk, int32_t* sel_ids, int32_t* sel_counts,
                           int32_t* pr_ids, int32_t* pr_counts, cudaStream_t stream) {
  const int rows = Hkv * Nt;
  if (rows == 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (rows * 32 + threads - 1) / threads;
  compact_kernel<<<blocks, threads, 0, stream>>>(mask, rows, Nt, Nb, block_k, tile_q, offset,
                                                 valid_lk, sel_ids, sel_counts, pr_ids, pr_counts);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_attn_generic(const AttnArgs& a, cudaStream_t stream) {
  const long long rows = (long long)a.Hq * a.Lq_pad;
  if (rows == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((rows + kAttnWarps - 1) / kAttnWarps);
  const size_t smem = sizeof(float) * kAttnWarps * a.D;
  if (a.dt == DT_BF16)
    attn_generic_kernel<DT_BF16><<<blocks, kAttnWarps * 32, smem, stream>>>(a);
  else if (a.dt == DT_F16)
    attn_generic_kernel<DT_F16><<<blocks, kAttnWarps * 32, smem, stream>>>(a);
  else
    return cudaErrorInvalidValue;
  count_launch();
  return cudaGetLastError();
}

}  // namespace fpv2
