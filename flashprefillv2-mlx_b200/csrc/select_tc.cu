// Index stage on tensor cores: scores, tile energies, alpha threshold,
// forcing and list compaction for one (KV head, query tile) per work item.
//
// Math (fpv2/selection.py:144-195, fpv2/kernel.py:170-183):
//   s[r, b]  = scale * q[r] . kbar[b]                 r over the tile's G*tile_q packed rows
//   M        = max over visible rows r and fully visible blocks b of s[r, b]
//   E[b]     = sum_r exp(s[r, b] - M)                 fully visible blocks only, else 0
//   sel[b]   = E[b] >= alpha * max_b E[b]
//   mask[b]  = (sel | sink | local | dense_tail) & visible
// The tensor cores compute the transposed score tile S^T = Kbar . Q^T
// (M = 128 blocks per TMEM lane group, N = the tile's packed query rows), so a
// thread owns one block: its max m_b and sum e_b = sum_r 2^(x - m_b) (x = s*log2 e)
// are register-local. The tile max is then M = max_b m_b and
// E[b] = e_b * 2^(m_b - M): no cross-thread reduction touches the N*Nb scores.
//
// Warp roles (320 threads, one persistent CTA per SM):
//   warp 0  TMA producer: Q chunks [N x D] and pooled-K tiles [128 x D], 128B swizzle.
//           A pooled-K tile stays in its ring slot while the CTA keeps the same
//           KV head, so pooled K is read from L2 once per CTA when Nb <= 128*slots.
//   warp 1  MMA issuer (tcgen05.mma kind::f16, fp32 accumulators in TMEM).
//   warps 2-5, 6-9  two energy + finalize groups: TMEM -> registers, masked
//           max / exp2-sums, then threshold, forcing and ballot-based
//           compaction into the full-width padded lists. The groups take a
//           CTA's items alternately (each owns two TMEM slots and its own
//           statistics), so one group's finalize overlaps the other group's
//           exponentials and each SM sub-partition has two warps issuing ex2.
// Work items are (kv head, tile) with tiles latest-first; CTA c keeps KV head
// c % Hkv whenever the grid is a multiple of Hkv.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace fpv2 {

namespace {

constexpr int kGroups = 2;           // energy/finalize warp groups
constexpr int kThreads = 64 + kGroups * 128;
constexpr int kTmemCols = 512;
constexpr int kTmemSlots = 4;        // 128 columns each
constexpr int kSlotsPerGroup = kTmemSlots / kGroups;
constexpr int kMaxNb = 2048;
constexpr int kSmemLimit = 227 * 1024;

template <int D>
struct Cfg {
  static constexpr int kHalves = D / 64;
  static constexpr int kQStages = (D == 256) ? 1 : 2;   // a 256-wide Q chunk is 64 KB
  static constexpr int kKStagesMax = (D == 64) ? 8 : (D == 256 ? 2 : 4);   // pooled-K ring (runtime count)
  static constexpr int kQBytes = 128 * D * 2;   // up to 128 rows per chunk
  static constexpr int kKBytes = 128 * D * 2;
};

struct Params {
  SelectGeom g;
  int NC, box_rows, n_chunks;
  int k_stages;                      // pooled-K ring slots in use (<= kKStagesMax)
  int nparts;                        // 16-bit parts of the pooled keys (3: float32 pooled K)
  const int* k_exp;                  // nparts == 3: per-KV-head exponent of the parts, else null
  uint32_t idesc;
  float scale_log2;
  uint8_t* mask;
  int32_t* sel_ids;
  int32_t* sel_counts;
  int32_t* pr_ids;
  int32_t* pr_counts;
  int* status;
  long long budget;
};

struct Item {
  int h, t;
  long long tile_first, tile_last;
  int n_full, n_mt;
  bool row_mask;   // some (row, fully visible block) pair needs a per-element test
};

__device__ __forceinline__ Item make_item(const Params& p, int w) {
  const SelectGeom& g = p.g;
  Item it;
  // (unsigned 32-bit divisions: every role derives each item's geometry on its
  // own critical path, and end <= offset + valid_lq < 2^32 always fits)
  it.h = (int)((unsigned)w % (unsigned)g.Hkv);
  it.t = g.Nt - 1 - (int)((unsigned)w / (unsigned)g.Hkv);
  it.tile_first = (long long)g.offset + (long long)it.t * g.tile_q;
  it.tile_last = min(it.tile_first + g.tile_q, (long long)g.offset + g.valid_lq) - 1;
  it.n_full = 0;
  const long long end = it.tile_last + 1;
  if (end >= g.block_k)
    it.n_full = (int)min((unsigned)g.Nb, (unsigned)end / (unsigned)g.block_k);
  it.n_mt = (it.n_full + 127) / 128;
  const bool all_rows_valid = (long long)(it.t + 1) * g.tile_q <= g.valid_lq;
  const bool all_see_all =
      it.n_full == 0 || (long long)(it.n_full - 1) * g.block_k <= it.tile_first;
  it.row_mask = !(all_rows_valid && all_see_all);
  return it;
}

// Order-preserving float <-> uint32 encoding (for atomicMax on floats).
__device__ __forceinline__ uint32_t f2ord(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Bits [0, n) of a 32-bit word (n clamped to [0, 32]).
__device__ __forceinline__ uint32_t prefix_bits(long long n) {
  return n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// kContig: each query chunk holds consecutive positions of one head (tile_q a
// multiple of the chunk width), so element masks are column ranges.
template <int D, bool kContig>
__global__ void __launch_bounds__(kThreads, 1)
    select_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_k, Params p) {
  using C = Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);
  const SelectGeom& g = p.g;
  const int Nb = g.Nb;
  const int nwords = (Nb + 31) / 32;

  // ---- shared memory carve-up -------------------------------------------
  const int KS = p.k_stages;
  const uint32_t q_smem = base;
  const uint32_t k_smem = base + C::kQStages * C::kQBytes;
  // per energy group: stats [Nb], selected / pruned words and their prefixes [nwords]
  float2* stats_all = reinterpret_cast<float2*>(gbase + C::kQStages * C::kQBytes +
                                                KS * C::kKBytes);      // [kGroups][Nb]
  uint32_t* words_all = reinterpret_cast<uint32_t*>(stats_all + kGroups * Nb);  // [kGroups][4][nwords]
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(words_all + kGroups * 4 * nwords) + 7) & ~uintptr_t(7));
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + C::kQStages;
  uint64_t* k_full = q_empty + C::kQStages;
  uint64_t* k_empty = k_full + C::kKStagesMax;
  uint64_t* t_full = k_empty + C::kKStagesMax;
  uint64_t* t_empty = t_full + kTmemSlots;
  uint64_t* drain = t_empty + kTmemSlots;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* sred_all = tmem_slot + 2;                      // [kGroups][2] ordered-int M, K
  int* totals_all = reinterpret_cast<int*>(sred_all + 2 * kGroups);   // [kGroups][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kQStages; ++i) {
      mbar_init(smem_u32(&q_full[i]), 1);
      mbar_init(smem_u32(&q_empty[i]), 1);
    }
    for (int i = 0; i < C::kKStagesMax; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
    }
    for (int i = 0; i < kTmemSlots; ++i) {
      mbar_init(smem_u32(&t_full[i]), 1);
      mbar_init(smem_u32(&t_empty[i]), 4);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  WaitCtx wc{p.status, abort_flag, p.budget};
  const int total_work = g.Hkv * g.Nt;
  // Tiles of several query chunks: the producer and the issuer walk two items
  // (one per energy group) together, alternating their score tiles, so both
  // groups stay busy. The same schedule serves single-chunk tiles whose pooled
  // keys outgrow the ring (Nb > 128 * slots): their tiles are reloaded for every
  // item, and two items walked together share each load (c5, 128k: index stage
  // 2.79 ms against 2.88; where the tiles stay resident it measured no gain).
  // (A 256-wide Q chunk has a single stage: one item at a time.)
  const bool k_reloaded = (g.Nb + 127) / 128 > KS;
  const int npair = (C::kQStages >= 2 && (p.n_chunks > 1 || k_reloaded)) ? 2 : 1;

  if (warp == 0) {
    // ======================= TMA producer =================================
    if (lane == 0) {
      int qcount = 0;
      int kuse[C::kKStagesMax];
      int ktag[C::kKStagesMax];
#pragma unroll
      for (int i = 0; i < C::kKStagesMax; ++i) { kuse[i] = 0; ktag[i] = -1; }
      bool ok = true;
      if (npair == 1) {
        for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x) {
          const Item it = make_item(p, w);
          if (it.n_mt == 0) continue;
          for (int c = 0; c < p.n_chunks && ok; ++c) {
            const int qs = qcount % C::kQStages;
            ok = mbar_wait(smem_u32(&q_empty[qs]), ((qcount / C::kQStages) & 1) ^ 1, wc);
            if (!ok) break;
            ++qcount;
            const uint32_t qb = smem_u32(&q_full[qs]);
            mbar_arrive_expect_tx(qb, (uint32_t)(p.NC * D * 2));
            const int P0 = c * p.NC;
            const int g0 = P0 / g.tile_q, p0 = P0 % g.tile_q;
  #pragma unroll
            for (int hh = 0; hh < C::kHalves; ++hh)
              tma_load_3d(q_smem + qs * C::kQBytes + hh * p.NC * 128, &tmap_q, qb, hh * 64,
                          it.t * g.tile_q + p0, it.h * g.G + g0);
            for (int mi = 0; mi < it.n_mt * p.nparts; ++mi) {   // (tile, part) pairs
              const int m = mi / p.nparts, part = mi % p.nparts;
              const int s = mi % KS;
              ok = mbar_wait(smem_u32(&k_empty[s]), (kuse[s] & 1) ^ 1, wc);
              if (!ok) break;
              ++kuse[s];
              const int tag = (it.h * 4096 + m) * 4 + part;
              const uint32_t kb = smem_u32(&k_full[s]);
              if (ktag[s] == tag) {
                mbar_arrive(kb);   // tile still resident
              } else {
                ktag[s] = tag;
                mbar_arrive_expect_tx(kb, (uint32_t)(128 * D * 2));
  #pragma unroll
                for (int hh = 0; hh < C::kHalves; ++hh)
                  tma_load_3d(k_smem + s * C::kKBytes + hh * 128 * 128, &tmap_k, kb, hh * 64, m * 128,
                              part * g.Hkv + it.h);
              }
            }
          }
        }
      } else {
        for (int w = blockIdx.x; w < total_work && ok; w += npair * gridDim.x) {
          Item its[2];
          int nmt[2] = {0, 0}, nmax = 0;
  #pragma unroll
          for (int x = 0; x < 2; ++x) {
            const int wx = w + x * gridDim.x;
            if (x < npair && wx < total_work) {
              its[x] = make_item(p, wx);
              nmt[x] = its[x].n_mt;
            }
            nmax = max(nmax, nmt[x]);
          }
          if (nmax == 0) continue;
          for (int c = 0; c < p.n_chunks && ok; ++c) {
  #pragma unroll
            for (int x = 0; x < 2; ++x) {
              if (nmt[x] == 0 || !ok) continue;
              const Item& it = its[x];
              const int qs = qcount % C::kQStages;
              ok = mbar_wait(smem_u32(&q_empty[qs]), ((qcount / C::kQStages) & 1) ^ 1, wc);
              if (!ok) break;
              ++qcount;
              const uint32_t qb = smem_u32(&q_full[qs]);
              mbar_arrive_expect_tx(qb, (uint32_t)(p.NC * D * 2));
              const int P0 = c * p.NC;
              const int g0 = P0 / g.tile_q, p0 = P0 % g.tile_q;
  #pragma unroll
              for (int hh = 0; hh < C::kHalves; ++hh)
                tma_load_3d(q_smem + qs * C::kQBytes + hh * p.NC * 128, &tmap_q, qb, hh * 64,
                            it.t * g.tile_q + p0, it.h * g.G + g0);
            }
            for (int mi = 0; mi < nmax * p.nparts && ok; ++mi) {   // (tile, part) pairs
              const int m = mi / p.nparts, part = mi % p.nparts;
  #pragma unroll
              for (int x = 0; x < 2; ++x) {
                if (m >= nmt[x] || !ok) continue;
                const int s = mi % KS;
                ok = mbar_wait(smem_u32(&k_empty[s]), (kuse[s] & 1) ^ 1, wc);
                if (!ok) break;
                ++kuse[s];
                const int tag = (its[x].h * 4096 + m) * 4 + part;
                const uint32_t kb = smem_u32(&k_full[s]);
                if (ktag[s] == tag) {
                  mbar_arrive(kb);   // tile still resident
                } else {
                  ktag[s] = tag;
                  mbar_arrive_expect_tx(kb, (uint32_t)(128 * D * 2));
  #pragma unroll
                  for (int hh = 0; hh < C::kHalves; ++hh)
                    tma_load_3d(k_smem + s * C::kKBytes + hh * 128 * 128, &tmap_k, kb, hh * 64, m * 128,
                                part * g.Hkv + its[x].h);
                }
              }
            }
          }
        }
      }
      // Drain: wait (bounded) for every armed barrier phase so no bulk copy is
      // still writing shared memory when the CTA retires.
      for (int i = 0; i < KS; ++i)
        if (kuse[i] > 0) mbar_wait(smem_u32(&k_full[i]), (kuse[i] - 1) & 1, wc, false);
      for (int i = 0; i < C::kQStages && i < qcount; ++i) {
        const int uses = (qcount - i + C::kQStages - 1) / C::kQStages;
        mbar_wait(smem_u32(&q_full[i]), (uses - 1) & 1, wc, false);
      }
    }
  } else if (warp == 1) {
    // ======================= MMA issuer ===================================
    if (lane == 0) {
      int qcount = 0;
      int tcount[kGroups] = {0, 0};
      int kuse[C::kKStagesMax];
#pragma unroll
      for (int i = 0; i < C::kKStagesMax; ++i) kuse[i] = 0;
      bool ok = true;
      int j = 0;   // CTA-local item index: item j belongs to energy group j % kGroups
      if (npair == 1) {
        for (int w = blockIdx.x; w < total_work && ok; w += gridDim.x, ++j) {
          const Item it = make_item(p, w);
          if (it.n_mt == 0) continue;
          const int grp = j % kGroups;
          for (int c = 0; c < p.n_chunks && ok; ++c) {
            const int qs = qcount % C::kQStages;
            ok = mbar_wait(smem_u32(&q_full[qs]), (qcount / C::kQStages) & 1, wc);
            if (!ok) break;
            ++qcount;
            for (int m = 0; m < it.n_mt && ok; ++m) {
              int ts = 0;
              // one score tile per m: the parts of the pooled keys accumulate into it
              for (int part = 0; part < p.nparts && ok; ++part) {
                const int s = (m * p.nparts + part) % KS;
                ok = mbar_wait(smem_u32(&k_full[s]), kuse[s] & 1, wc);
                if (!ok) break;
                ++kuse[s];
                if (part == 0) {
                  const int tc = tcount[grp];
                  ts = grp * kSlotsPerGroup + tc % kSlotsPerGroup;
                  ok = mbar_wait(smem_u32(&t_empty[ts]), ((tc / kSlotsPerGroup) & 1) ^ 1, wc);
                  if (!ok) break;
                  ++tcount[grp];
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + ts * 128;
  #pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                  const int hh = kk / 4, sub = kk % 4;
                  const uint64_t a_desc =
                      sw128_desc(k_smem + s * C::kKBytes + hh * 128 * 128 + sub * 32, 16, 1024);
                  const uint64_t b_desc =
                      sw128_desc(q_smem + qs * C::kQBytes + hh * p.NC * 128 + sub * 32, 16, 1024);
                  umma_ss(d_tmem, a_desc, b_desc, p.idesc, (part > 0 || kk > 0) ? 1u : 0u);
                }
                if (part == p.nparts - 1) umma_commit(smem_u32(&t_full[ts]));
                umma_commit(smem_u32(&k_empty[s]));
              }
            }
            if (ok) umma_commit(smem_u32(&q_empty[qs]));
          }
        }
      } else {
        for (int w = blockIdx.x; w < total_work && ok; w += npair * gridDim.x, j += npair) {
          int nmt[2] = {0, 0}, nmax = 0;
  #pragma unroll
          for (int x = 0; x < 2; ++x) {
            const int wx = w + x * gridDim.x;
            if (x < npair && wx < total_work) nmt[x] = make_item(p, wx).n_mt;
            nmax = max(nmax, nmt[x]);
          }
          if (nmax == 0) continue;
          for (int c = 0; c < p.n_chunks && ok; ++c) {
            int qsx[2] = {0, 0};
  #pragma unroll
            for (int x = 0; x < 2; ++x) {
              if (nmt[x] == 0 || !ok) continue;
              qsx[x] = qcount % C::kQStages;
              ok = mbar_wait(smem_u32(&q_full[qsx[x]]), (qcount / C::kQStages) & 1, wc);
              ++qcount;
            }
            // (tile, part) pairs in the producer's order; the parts of one tile
            // accumulate into one score tile of each item
            int tsx[2] = {0, 0};
            for (int mi = 0; mi < nmax * p.nparts && ok; ++mi) {
              const int m = mi / p.nparts, part = mi % p.nparts;
  #pragma unroll
              for (int x = 0; x < 2; ++x) {
                if (m >= nmt[x] || !ok) continue;
                const int grp = (j + x) % kGroups;
                const int s = mi % KS;
                ok = mbar_wait(smem_u32(&k_full[s]), kuse[s] & 1, wc);
                if (!ok) break;
                ++kuse[s];
                if (part == 0) {
                  const int tc = tcount[grp];
                  tsx[x] = grp * kSlotsPerGroup + tc % kSlotsPerGroup;
                  ok = mbar_wait(smem_u32(&t_empty[tsx[x]]), ((tc / kSlotsPerGroup) & 1) ^ 1, wc);
                  if (!ok) break;
                  ++tcount[grp];
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + tsx[x] * 128;
                const uint32_t qsm = q_smem + qsx[x] * C::kQBytes;
  #pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                  const int hh = kk / 4, sub = kk % 4;
                  const uint64_t a_desc =
                      sw128_desc(k_smem + s * C::kKBytes + hh * 128 * 128 + sub * 32, 16, 1024);
                  const uint64_t b_desc = sw128_desc(qsm + hh * p.NC * 128 + sub * 32, 16, 1024);
                  umma_ss(d_tmem, a_desc, b_desc, p.idesc, (part > 0 || kk > 0) ? 1u : 0u);
                }
                if (part == p.nparts - 1) umma_commit(smem_u32(&t_full[tsx[x]]));
                umma_commit(smem_u32(&k_empty[s]));
                // this item's query chunk is read for the last time
                if (m == nmt[x] - 1 && part == p.nparts - 1) umma_commit(smem_u32(&q_empty[qsx[x]]));
              }
            }
          }
        }
      }
      // Drain: every MMA issued by this thread has completed once `drain` flips.
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, wc, false);
    }
  } else {
    // ======================= energy + finalize =============================
    // Thread (quarter, lane) owns block b = 128 m + 32 quarter + lane of every
    // M-tile m: m_b = max over the tile's visible rows of x = s * log2(e), and
    // e_b = sum_rows 2^(x - m_b). The tile max M = max_b m_b and the energy max
    // 2^(K - M) with K = max_b (m_b + log2 e_b) are reduced with shared-memory
    // atomics on order-preserving integer encodings while the tiles stream by.
    const int grp = (warp - 2) >> 2;          // energy group of this warp
    const int et = threadIdx.x - 64 - grp * 128;   // 0..127 within the group
    const int quarter = warp & 3;              // TMEM lane group of this warp
    const int ew = et >> 5;                    // 0..3 index among the group's warps
    const int bar_id = 1 + grp;                // the group's named barrier
    const unsigned lt = (1u << lane) - 1u;
    float2* stats = stats_all + grp * Nb;
    uint32_t* selw = words_all + grp * 4 * nwords;
    uint32_t* prw = selw + nwords;
    int* selpre = reinterpret_cast<int*>(prw + nwords);
    int* prpre = selpre + nwords;
    uint32_t* sred = sred_all + 2 * grp;
    int* totals = totals_all + 2 * grp;
    int tcount = 0;
    bool ok = true;   // after a failed wait the role keeps its barrier schedule but skips TMEM
    if (et == 0) {
      sred[0] = f2ord(-INFINITY);
      sred[1] = f2ord(-INFINITY);
    }
    named_bar_sync(bar_id, 128);
    for (int w = blockIdx.x + grp * gridDim.x; w < total_work; w += kGroups * gridDim.x) {
      const Item it = make_item(p, w);
      // > 0 on this path; float32 pooled keys of a head scaled by 2^-e score at 2^e
      const float c = p.k_exp == nullptr ? p.scale_log2 : ldexpf(p.scale_log2, p.k_exp[it.h]);
      const long long row_base = ((long long)it.h * g.Nt + it.t) * Nb;
      for (int cc = 0; cc < p.n_chunks; ++cc) {
        for (int m = 0; m < it.n_mt; ++m) {
          const int ts = grp * kSlotsPerGroup + tcount % kSlotsPerGroup;
          if (ok) ok = mbar_wait(smem_u32(&t_full[ts]), (tcount / kSlotsPerGroup) & 1, wc);
          ok = __all_sync(0xffffffffu, ok);   // the TMEM loads below are warp-collective
          ++tcount;
          tc_fence_after();
          const int b = m * 128 + quarter * 32 + lane;
          if (ok && m * 128 + quarter * 32 < it.n_full) {
            const bool bvalid = b < it.n_full;
            float mb = -INFINITY, eb = 0.f;
            if (cc > 0 && bvalid) {
              const float2 st = stats[b];
              mb = st.x;
              eb = st.y;
            }
            // Two passes of 64 columns (registers: the CTA runs 10 warps, so a
            // thread has at most 168); (m_b, e_b) is carried online between them.
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + ts * 128;
            // Element masks are needed only for partially visible rows or a
            // narrow N-chunk; the decision is per item, so it never diverges
            // inside a warp. Lanes past the fully visible blocks compute on
            // whatever the tile holds and are simply not recorded.
            const bool masked = it.row_mask || p.NC < 128;
            const long long bstart = (long long)b * g.block_k;
#pragma unroll 1
            for (int hf = 0; hf < 2; ++hf) {
              if (hf * 64 >= p.NC) break;
              uint32_t sv[2][32];
              tmem_ld32(taddr + hf * 64, sv[0]);
              if (hf * 64 + 32 < p.NC) tmem_ld32(taddr + hf * 64 + 32, sv[1]);
              tmem_wait_ld();
              reg_fence(sv[0]);
              reg_fence(sv[1]);
              uint32_t vm[2] = {0xffffffffu, 0xffffffffu};
              if (kContig && masked) {
                // The chunk's columns are consecutive positions row0 + col: the
                // visible columns of block b form the range [lo, hi).
                const long long row0 = (long long)it.t * g.tile_q + (cc * p.NC) % g.tile_q;
                long long lo = 0, hi = p.NC;
                if (it.row_mask) {
                  lo = max(lo, bstart - g.offset - row0);            // bstart <= offset + row
                  hi = min(hi, (long long)g.valid_lq - row0);         // row < valid_lq
                }
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                  const long long c0 = hf * 64 + q2 * 32;
                  vm[q2] = prefix_bits(hi - c0) & ~prefix_bits(lo - c0);
                }
              } else if (masked) {
#pragma unroll 1
                for (int q2 = 0; q2 < 2; ++q2) {
                  uint32_t bits = 0u;
                  for (int j = 0; j < 32; ++j) {
                    const int col = hf * 64 + q2 * 32 + j;
                    bool v = col < p.NC;
                    if (v && it.row_mask) {
                      const int P = cc * p.NC + col;
                      const long long row = (long long)it.t * g.tile_q + P % g.tile_q;
                      v = row < g.valid_lq && bstart <= g.offset + row;
                    }
                    bits |= v ? (1u << j) : 0u;
                  }
                  vm[q2] = bits;
                }
              }
              // Masked-out entries become -inf: they drop out of the max and
              // 2^(-inf) = 0 drops them from the sum.
              if (masked) {
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                  sv[0][j] = ((vm[0] >> j) & 1u) ? sv[0][j] : 0xff800000u;
                  sv[1][j] = ((vm[1] >> j) & 1u) ? sv[1][j] : 0xff800000u;
                }
              }
              float m0 = max3f(__uint_as_float(sv[0][0]), __uint_as_float(sv[0][1]), __uint_as_float(sv[0][2]));
              float m1 = max3f(__uint_as_float(sv[0][16]), __uint_as_float(sv[0][17]), __uint_as_float(sv[0][18]));
              float m2 = max3f(__uint_as_float(sv[1][0]), __uint_as_float(sv[1][1]), __uint_as_float(sv[1][2]));
              float m3 = max3f(__uint_as_float(sv[1][16]), __uint_as_float(sv[1][17]), __uint_as_float(sv[1][18]));
#pragma unroll
              for (int j = 3; j < 15; j += 2) {
                m0 = max3f(m0, __uint_as_float(sv[0][j]), __uint_as_float(sv[0][j + 1]));
                m1 = max3f(m1, __uint_as_float(sv[0][16 + j]), __uint_as_float(sv[0][17 + j]));
                m2 = max3f(m2, __uint_as_float(sv[1][j]), __uint_as_float(sv[1][j + 1]));
                m3 = max3f(m3, __uint_as_float(sv[1][16 + j]), __uint_as_float(sv[1][17 + j]));
              }
              m0 = max3f(m0, __uint_as_float(sv[0][15]), m1);
              m2 = max3f(m2, __uint_as_float(sv[1][15]), m3);
              const float mraw = max3f(m0, m2, fmaxf(__uint_as_float(sv[0][31]), __uint_as_float(sv[1][31])));
              const float mnew = fmaxf(mb, mraw * c);
              // all lanes take the same path below (-inf maxima give ex2(-inf) = 0)
              const float nm = mnew == -INFINITY ? 0.f : -mnew;
              // pairs of scores: one packed FMA forms both exponents, packed adds sum;
              // a quarter of the exponentials run on the FMA pipe (relative error
              // < 2.7e-6, well inside the 1e-5 band in which a block may flip)
              const float2 c2 = make_float2(c, c), nm2 = make_float2(nm, nm);
              float2 e[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                             make_float2(0.f, 0.f)};
#pragma unroll
              for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                  const float2 xv = fma_f32x2(
                      make_float2(__uint_as_float(sv[h2][j]), __uint_as_float(sv[h2][j + 1])), c2, nm2);
                  const float2 pv = ((j >> 1) & 3) == 3 ? exp2_poly_x2(xv) : make_float2(ex2(xv.x), ex2(xv.y));
                  e[(j >> 1) & 3] = add_f32x2(e[(j >> 1) & 3], pv);
                }
              const float esum = ((e[0].x + e[0].y) + (e[1].x + e[1].y)) + ((e[2].x + e[2].y) + (e[3].x + e[3].y));
              if (mnew != -INFINITY) {
                eb = eb * ex2(mb - mnew) + esum;
                mb = mnew;
              }
            }
            if (bvalid) stats[b] = make_float2(mb, eb);
            if (cc == p.n_chunks - 1) {
              // fold this block into the tile max M and the energy-max key K
              float wm = bvalid ? mb : -INFINITY;
              float wk = (bvalid && eb > 0.f) ? mb + lg2(eb) : -INFINITY;
              wm = warp_max(wm);
              wk = warp_max(wk);
              if (lane == 0) {
                atomicMax(&sred[0], f2ord(wm));
                atomicMax(&sred[1], f2ord(wk));
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&t_empty[ts]));
        }
      }

      // ---- finalize: threshold, forcing, lists ----------------------------
      named_bar_sync(bar_id, 128);                 // stats, M and K complete
      const float Mx = ord2f(sred[0]);
      const float Kx = ord2f(sred[1]);
      const float emax = (Mx == -INFINITY || Kx == -INFINITY) ? 0.f : ex2(Kx - Mx);
      const float thr = g.alpha * emax;
      const bool dense_tail = it.t >= max(g.Nt - g.last_n, 0);
      // (unrolled: the statistics loads and exponentials of four word groups
      // are independent, so their latencies overlap)
#pragma unroll 4
      for (int base_b = ew * 32; base_b < Nb; base_b += 128) {
        const int b = base_b + lane;
        const long long bs = (long long)b * g.block_k, be = bs + g.block_k;
        float E = 0.f;
        if (b < it.n_full) {
          const float2 st = stats[b];
          E = (Mx == -INFINITY || st.x == -INFINITY) ? 0.f : st.y * ex2(st.x - Mx);
        }
        const bool forced = bs < g.sink || be > it.tile_first - g.window || dense_tail;
        const bool fin = b < Nb && (E >= thr || forced) && bs <= it.tile_last;
        const bool pr = b < Nb && !fin && min(be, (long long)g.valid_lk) <= it.tile_first;
        const unsigned sb = __ballot_sync(0xffffffffu, fin);
        const unsigned pb = __ballot_sync(0xffffffffu, pr);
        if (lane == 0) {
          selw[base_b >> 5] = sb;
          prw[base_b >> 5] = pb;
        }
        if (p.mask != nullptr && b < Nb) p.mask[row_base + b] = (uint8_t)fin;
      }
      named_bar_sync(bar_id, 128);                 // words complete; M, K consumed
      if (et == 0) {
        sred[0] = f2ord(-INFINITY);
        sred[1] = f2ord(-INFINITY);
      }
      if (p.sel_ids != nullptr && ew == 0) {
        int run_s = 0, run_p = 0;
        for (int w0 = 0; w0 < nwords; w0 += 32) {
          const int wi = w0 + lane;
          const int cs = wi < nwords ? __popc(selw[wi]) : 0;
          const int cp = wi < nwords ? __popc(prw[wi]) : 0;
          int is = cs, ip = cp;   // inclusive warp scan
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int ys = __shfl_up_sync(0xffffffffu, is, o);
            const int yp = __shfl_up_sync(0xffffffffu, ip, o);
            if (lane >= o) { is += ys; ip += yp; }
          }
          if (wi < nwords) {
            selpre[wi] = run_s + is - cs;
            prpre[wi] = run_p + ip - cp;
          }
          run_s += __shfl_sync(0xffffffffu, is, 31);
          run_p += __shfl_sync(0xffffffffu, ip, 31);
        }
        if (lane == 0) {
          totals[0] = run_s;
          totals[1] = run_p;
        }
      }
      named_bar_sync(bar_id, 128);                 // prefixes complete
      if (p.sel_ids != nullptr) {
        const int nsel = totals[0], npr = totals[1];
#pragma unroll 4
        for (int base_b = ew * 32; base_b < Nb; base_b += 128) {
          const int b = base_b + lane;
          if (b < Nb) {
            const int wi = base_b >> 5;
            const uint32_t sb = selw[wi], pb = prw[wi];
            const int rs = selpre[wi] + __popc(sb & lt);
            const int rp = prpre[wi] + __popc(pb & lt);
            p.sel_ids[row_base + (((sb >> lane) & 1u) ? rs : nsel + (b - rs))] = b;
            p.pr_ids[row_base + (((pb >> lane) & 1u) ? rp : npr + (b - rp))] = b;
          }
        }
        if (et == 0) {
          p.sel_counts[(long long)it.h * g.Nt + it.t] = nsel;
          p.pr_counts[(long long)it.h * g.Nt + it.t] = npr;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

template <int D>
size_t smem_bytes(int Nb, int k_stages) {
  const int nwords = (Nb + 31) / 32;
  size_t s = 1024 + (size_t)Cfg<D>::kQStages * Cfg<D>::kQBytes + (size_t)k_stages * Cfg<D>::kKBytes;
  s += (size_t)kGroups * ((size_t)Nb * 8 + (size_t)nwords * 16);
  s += 8 + 8 * (2 * Cfg<D>::kQStages + 2 * Cfg<D>::kKStagesMax + 2 * kTmemSlots + 1);
  s += 8 + 16 * kGroups + 8;
  return s;
}

// Largest pooled-K ring that fits next to the per-group statistics (0 if < 2).
template <int D>
int pick_k_stages(int Nb) {
  for (int ks = Cfg<D>::kKStagesMax; ks >= 2; --ks)
    if (smem_bytes<D>(Nb, ks) <= (size_t)kSmemLimit) return ks;
  return 0;
}

}  // namespace

bool select_tc_supported(const SelectGeom& g, int dt) {
  if (dt != DT_BF16 && dt != DT_F16) return false;
  if (!(g.scale > 0.f)) return false;
  if (g.D != 64 && g.D != 96 && g.D != 128 && g.D != 256) return false;   // 96: zero-padded 128-wide tiles
  if (g.Nb > kMaxNb || g.Nb <= 0) return false;
  const int ks = g.D == 64 ? pick_k_stages<64>(g.Nb)
                 : (g.D == 256 ? pick_k_stages<256>(g.Nb) : pick_k_stages<128>(g.Nb));
  if (ks == 0) return false;
  const int R = g.G * g.tile_q;
  if (R >= 128) {
    if (R % 128) return false;
    if (g.tile_q % 128 != 0 && 128 % g.tile_q != 0) return false;
  } else {
    if (R % 16) return false;
  }
  if (g.tile_q > 256) return g.tile_q % 128 == 0;
  return true;
}

cudaError_t launch_select_tc(const SelectTcArgs& a, const void* q, const void* pk,
                             const TcLaunch& L, cudaStream_t stream) {
  const SelectGeom& g = a.g;
  Params p;
  p.g = g;
  p.NC = a.NC;
  p.box_rows = a.box_rows;
  p.n_chunks = (g.G * g.tile_q) / a.NC;
  p.idesc = umma_idesc_f16(a.dt == DT_BF16 ? 1 : 0, 128, a.NC, 0, 0);
  p.scale_log2 = g.scale * kLog2e;
  p.mask = a.mask;
  p.sel_ids = a.sel_ids;
  p.sel_counts = a.sel_counts;
  p.pr_ids = a.pr_ids;
  p.pr_counts = a.pr_counts;
  p.status = L.status;
  p.budget = L.budget;
  p.nparts = a.nparts;
  p.k_exp = a.k_exp;

  CUtensorMap tq, tk;
  if (!encode_tmap_3d(&tq, q, a.dt, (uint64_t)g.D, (uint64_t)g.Lq_pad, (uint64_t)g.Hq, 64,
                      (uint32_t)a.box_rows, (uint32_t)a.box_heads))
    return cudaErrorInvalidValue;
  // (pooled keys [nparts][Hkv][Nb][D]: part p of head h is "head" p * Hkv + h)
  if (!encode_tmap_3d(&tk, pk, a.dt, (uint64_t)g.D, (uint64_t)g.Nb, (uint64_t)g.Hkv * a.nparts, 64,
                      128, 1))
    return cudaErrorInvalidValue;

  const int total = g.Hkv * g.Nt;
  int grid;
  if (g.Hkv <= L.num_sms) {
    const int per_head = max(1, min(L.num_sms / g.Hkv, g.Nt));
    grid = per_head * g.Hkv;
  } else {
    grid = L.num_sms;
  }
  grid = max(1, min(grid, total));
  const bool contig = g.tile_q % a.NC == 0;
  cudaError_t e;
#define FPV2_SELECT_LAUNCH(DD)                                                                 \
  {                                                                                            \
    p.k_stages = pick_k_stages<DD>(g.Nb);                                                      \
    const size_t smem = smem_bytes<DD>(g.Nb, p.k_stages);                                      \
    auto kern = contig ? select_tc_kernel<DD, true> : select_tc_kernel<DD, false>;             \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);    \
    if (e != cudaSuccess) return e;                                                            \
    kern<<<grid, kThreads, smem, stream>>>(tq, tk, p);                                         \
    count_launch();                                                                            \
  }
  if (g.D == 64) FPV2_SELECT_LAUNCH(64)
  else if (g.D == 256) FPV2_SELECT_LAUNCH(256)
  else FPV2_SELECT_LAUNCH(128)
#undef FPV2_SELECT_LAUNCH
  return cudaGetLastError();
}

namespace {

constexpr size_t up_to(size_t x, size_t a) { return (x + a - 1) / a * a; }

// float32 pooled keys -> three 16-bit parts, out[p][i] for p = 0, 1, 2:
// round(y), round(y - part0), round(y - part0 - part1) with y = x * 2^-e[h].
// Their sum carries about 24 (bf16) or 33 (fp16) significant bits, so Q.K^T
// accumulated over the parts in fp32 equals the float32 product to within
// float32 rounding (fp16 parts of magnitudes below 2^-14 keep an absolute
// precision of 2^-25). e[h] >= 0 is the smallest exponent that brings KV head
// h's largest magnitude within the 16-bit type's range: 0 for any pooled keys
// of 16-bit inputs, and 0 for non-finite maxima (which score as in float32);
// the selection kernel scores head h at scale * 2^e[h].
//
// pk_absmax_kernel: grid (blocks, Hkv), the heads' maximum magnitudes as
// order-preserving bit patterns (non-negative floats order as integers).
__global__ void __launch_bounds__(256) pk_absmax_kernel(const float* __restrict__ pk,
                                                        unsigned* amax, long long per_head) {
  const int h = blockIdx.y;
  const float* src = pk + (long long)h * per_head;
  float m = 0.f;
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < per_head;
       i += (long long)gridDim.x * 256)
    m = fmaxf(m, fabsf(src[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(&amax[h], __float_as_uint(m));
}

// Smallest e >= 0 with amax * 2^-e <= limit (0 for non-finite or in-range maxima).
__device__ __forceinline__ int range_exponent(float amax, float limit) {
  if (!(amax > limit) || !(amax <= 3.402823466e38f)) return 0;
  int e = ilogbf(amax) - ilogbf(limit);
  if (ldexpf(amax, -e) > limit) ++e;
  return e;
}

template <int DT>
__global__ void __launch_bounds__(256) pk_split3_kernel(const float* __restrict__ pk, void* out,
                                                        const unsigned* __restrict__ amax,
                                                        int* k_exp, int Hkv, long long per_head) {
  using T = typename Elem<DT>::T;
  // largest finite magnitude of the part type
  const float limit = DT == DT_F16 ? 65504.f : 3.38953139e38f;
  T* o = reinterpret_cast<T*>(out);
  const long long n = (long long)Hkv * per_head;
  if (blockIdx.x == 0)
    for (int h = threadIdx.x; h < Hkv; h += 256) k_exp[h] = range_exponent(__uint_as_float(amax[h]), limit);
  for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n; i += (long long)gridDim.x * 256) {
    const int e = range_exponent(__uint_as_float(amax[i / per_head]), limit);
    const float x = e ? ldexpf(pk[i], -e) : pk[i];
    const T h = Elem<DT>::from_f(x);
    const float r1 = x - Elem<DT>::to_f(h);
    const T m = Elem<DT>::from_f(r1);
    const float r2 = r1 - Elem<DT>::to_f(m);
    o[i] = h;
    o[n + i] = m;
    o[2 * n + i] = Elem<DT>::from_f(r2);
  }
}

}  // namespace

size_t pk_split3_bytes(int Hkv, int Nb, int D) {
  return up_to((size_t)3 * Hkv * Nb * D * 2, 256) + 2 * sizeof(int) * (size_t)Hkv;
}

cudaError_t launch_pk_split3(const float* pk, void* out, int dt, int Hkv, int Nb, int D,
                             const int** k_exp, cudaStream_t stream) {
  const long long per_head = (long long)Nb * D;
  const long long n = per_head * Hkv;
  unsigned* amax = reinterpret_cast<unsigned*>(static_cast<char*>(out) + up_to((size_t)3 * n * 2, 256));
  int* ex = reinterpret_cast<int*>(amax + Hkv);
  *k_exp = ex;
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(unsigned) * Hkv, stream);
  if (e != cudaSuccess) return e;
  const int gx = (int)std::max<long long>(1, std::min<long long>((per_head + 255) / 256, 64));
  pk_absmax_kernel<<<dim3(gx, Hkv), 256, 0, stream>>>(pk, amax, per_head);
  count_launch();
  const int grid = (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 4096));
  if (dt == DT_BF16)
    pk_split3_kernel<DT_BF16><<<grid, 256, 0, stream>>>(pk, out, amax, ex, Hkv, per_head);
  else if (dt == DT_F16)
    pk_split3_kernel<DT_F16><<<grid, 256, 0, stream>>>(pk, out, amax, ex, Hkv, per_head);
  else
    return cudaErrorInvalidValue;
  count_launch();
  return cudaGetLastError();
}

}  // namespace fpv2
