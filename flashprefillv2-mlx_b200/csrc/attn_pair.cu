// Block-sparse attention on tensor cores, two query chunks per K/V stream.
//
// Same math as attn_tc.cu (fpv2/kernel.py:187-414): an online softmax in base
// 2 over the keys of the selected blocks, then the pruned blocks as pooled
// K/V entries with their logits shifted by log2(block_k); out = O / l.
//
// The chunks of one selection tile that cover the same query positions (the
// G query heads of a KV head, packed 128 rows at a time) read exactly the
// same K/V tiles: same lists, same causal extent. This kernel takes such
// chunks in pairs (A, B) as one work item, so every K/V tile staged in shared
// memory feeds two QK and two PV products, and the two chunks' softmax runs
// alternate with each other's tensor work:
//   S_A = Q_A K^T  ->  softmax A  ->  O_A += P_A V
//   S_B = Q_B K^T  ->  softmax B  ->  O_B += P_B V
// issued as QK_A(k), PV_B(k-1), QK_B(k), PV_A(k), QK_A(k+1), ... so the
// tensor pipe works on one chunk while the other chunk's softmax runs.
// TMEM = O_A | O_B | S_A | S_B (4 x 128 columns); P overwrites the first
// columns of its S tile, and the next QK into that tile is issued after the
// PV that reads P (tcgen05.mma from one thread execute in issue order).
//
// Softmax: four warps per chunk, one query row per thread and all 128 keys of
// the S tile, one running max m and sum l per row, O rescaled lazily (only
// when m grows by more than 2^16, 2^15 for fp16). P of keys 0..63 is handed to
// the MMA issuer before keys 64..127 are exponentiated, so the first half of
// the PV product overlaps the second half of the softmax. The output rows
// are written straight from registers (no staging buffer), which frees a
// query tile's shared memory as soon as its last QK product has completed.
//
// Warp roles (320 threads, one persistent CTA per SM):
//   warp 0     producer: work items from a global counter (latest tiles
//              first), one record per KV item, TMA loads of Q / K / V /
//              pooled tiles (no multicast);
//   warp 1     MMA issuer;
//   warps 2-3  idle (they complete the first warpgroup, whose registers go to
//              the softmax warpgroups through setmaxnreg);
//   warps 4-7  softmax and output of chunk A (thread = row, lane quarter = warp % 4);
//   warps 8-11 the same for chunk B.
#include "attn_common.cuh"

#include <algorithm>

namespace fpv2 {

namespace {

constexpr int kThreads = 384;
// Registers per thread: 168 at launch (65536 / 384, rounded down to 8); the
// first warpgroup drops to 72 and the two softmax warpgroups rise to 216
// (72 * 128 + 216 * 256 = 168 * 384), enough to hold a 128-key S row.
constexpr int kRegsLow = 72;
constexpr int kRegsHigh = 216;
static_assert(kRegsLow * 128 + kRegsHigh * 256 <= 168 * kThreads, "register split");
constexpr int kStages = 2;      // K and V tiles
constexpr int kQSlots = 3;      // query tiles (two per work item, one loading ahead)
constexpr int kRecs = 8;
constexpr int kTmemCols = 512;

template <int D>
struct PCfg {
  static constexpr int kHalves = D / 64;
  static constexpr int kTileBytes = 128 * D * 2;
  static constexpr int kOCol = 0;      // O_A at 0, O_B at 128
  static constexpr int kSCol = 256;    // S_A at 256, S_B at 384
};

struct Pair {
  int h, t;
  int c[2];                 // chunk index inside the tile of A and B
  int g0[2], p0;            // first head of each chunk, first position (shared)
  long long abs_last;       // last valid absolute query position (shared)
};

// Chunks c = hg * cpg + pi (cpg = chunks per head group, pi = position slice):
// pair j joins head groups 2 hg' and 2 hg' + 1 at the same position slice.
__device__ __forceinline__ Pair make_pair(const Params& p, int w) {
  const AttnArgs& a = p.a;
  Pair pr;
  const int ppt = p.nch / 2;
  const int per_t = a.Hkv * ppt;
  pr.t = a.Nt - 1 - w / per_t;   // latest tiles (most causal work) first
  const int r = w % per_t;
  pr.h = r / ppt;
  const int j = r % ppt;
  const int cpg = a.tile_q >= 128 ? a.tile_q / 128 : 1;
  const int pi = j % cpg, hgp = j / cpg;
  pr.c[0] = 2 * hgp * cpg + pi;
  pr.c[1] = pr.c[0] + cpg;
  pr.g0[0] = pr.c[0] * 128 / a.tile_q;
  pr.g0[1] = pr.c[1] * 128 / a.tile_q;
  pr.p0 = (pr.c[0] * 128) % a.tile_q;
  const long long span = min(a.tile_q, 128);
  const long long last_row =
      min((long long)pr.t * a.tile_q + pr.p0 + span, (long long)a.valid_lq) - 1;
  pr.abs_last = (long long)a.offset + last_row;
  return pr;
}

// DT: input dtype; VT: operand type of the P.V product (V and P).
template <int D, int DT, int VT>
__global__ void __launch_bounds__(kThreads, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_k,
                     const __grid_constant__ CUtensorMap tmap_v,
                     const __grid_constant__ CUtensorMap tmap_pk,
                     const __grid_constant__ CUtensorMap tmap_pv, Params p) {
  using C = PCfg<D>;
  const AttnArgs& a = p.a;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);

  const uint32_t q_smem = base;                                   // [kQSlots][tile]
  const uint32_t k_smem = base + kQSlots * C::kTileBytes;         // [kStages][tile]
  const uint32_t v_smem = k_smem + kStages * C::kTileBytes;       // [kStages][tile]
  uint8_t* after_tiles = gbase + (kQSlots + 2 * kStages) * C::kTileBytes;
  Rec* recs = reinterpret_cast<Rec*>(after_tiles);                // [kRecs]
  uint32_t* pmask = reinterpret_cast<uint32_t*>(recs + kRecs);    // producer-private [64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(pmask + kMaskWordsMax);
  uint64_t* q_full = bars;                   // [kQSlots]
  uint64_t* q_empty = q_full + kQSlots;      // [kQSlots]
  uint64_t* rec_full = q_empty + kQSlots;    // [kRecs]
  uint64_t* rec_empty = rec_full + kRecs;    // [kRecs]
  uint64_t* k_full = rec_empty + kRecs;      // [kStages]
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;      // [2 chunk]
  uint64_t* p_full = s_full + 2;             // [2 chunk][2 key half] (4 warps each)
  uint64_t* pv_done = p_full + 4;            // [2 chunk]
  uint64_t* o_full = pv_done + 2;            // [2 chunk]
  uint64_t* drain = o_full + 2;              // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQSlots; ++i) {
      mbar_init(smem_u32(&q_full[i]), 1);
      mbar_init(smem_u32(&q_empty[i]), 1);   // the last QK reading the slot
    }
    for (int i = 0; i < kRecs; ++i) {
      mbar_init(smem_u32(&rec_full[i]), 1);
      mbar_init(smem_u32(&rec_empty[i]), 1 + 8);   // MMA thread + 8 softmax warps
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&k_full[i]), 1);
      mbar_init(smem_u32(&k_empty[i]), 1);
      mbar_init(smem_u32(&v_full[i]), 1);
      mbar_init(smem_u32(&v_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[2 * i]), 4);
      mbar_init(smem_u32(&p_full[2 * i + 1]), 4);
      mbar_init(smem_u32(&pv_done[i]), 1);
      mbar_init(smem_u32(&o_full[i]), 1);
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
    tma_prefetch_desc(&tmap_v);
    tma_prefetch_desc(&tmap_pk);
    tma_prefetch_desc(&tmap_pv);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  WaitCtx wc{p.status, abort_flag, p.budget};
  const int bk_sub = a.block_k / 128;
  const bool pool_tiles = a.corr && a.pooled_dt == DT;   // TMA pooled tiles vs gather

  if (warp < 4) {
  regs_dec<kRegsLow>();
  if (warp == 0) {
    // ============================ producer ================================
    int qcount = 0, icount = 0, kv = 0, wstatic = blockIdx.x;
    bool ok = true;
    auto next_work = [&]() -> int {
      int w = 0;
      if (p.sched != nullptr) {
        if (lane == 0) w = atomicAdd(p.sched, 1);
        w = __shfl_sync(0xffffffffu, w, 0);
      } else {
        w = wstatic;
        wstatic += gridDim.x;
      }
      return w;
    };
    // Publish one record; SEL/POOL/CORR records are followed by their K/V tiles.
    auto emit = [&](const Rec& rec, int h, long long lrow) -> bool {
      const int ri = icount % kRecs;
      bool good = true;
      if (lane == 0) good = mbar_wait(smem_u32(&rec_empty[ri]), ((icount / kRecs) & 1) ^ 1, wc);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) return false;
      if (lane == 0) {
        recs[ri] = rec;
        mbar_arrive(smem_u32(&rec_full[ri]));
      }
      ++icount;
      if (rec.kind == KIND_EMPTY || rec.kind == KIND_DONE) return true;
      const int st = kv % kStages;
      const uint32_t par = ((kv / kStages) & 1) ^ 1;
      const uint32_t kst = k_smem + st * C::kTileBytes;
      const uint32_t vst = v_smem + st * C::kTileBytes;
      if (rec.kind != KIND_CORR) {
        if (lane == 0) {
          const CUtensorMap* mk = rec.kind == KIND_SEL ? &tmap_k : &tmap_pk;
          const CUtensorMap* mv = rec.kind == KIND_SEL ? &tmap_v : &tmap_pv;
          // (a converted V copy is contiguous even when the page pools are not)
          const bool paged_k = rec.kind == KIND_SEL && a.block_table != nullptr;
          const bool paged_v = paged_k && a.v_conv == nullptr;
          // One 128-row tile: a 3-D box per 64 features, or, from a page pool,
          // one 4-D box per page the 128 keys span.
          auto load_tile = [&](uint32_t dst, const CUtensorMap* m, uint32_t bar, bool paged) {
            mbar_arrive_expect_tx(bar, (uint32_t)C::kTileBytes);
            if (!paged) {
#pragma unroll
              for (int hh = 0; hh < C::kHalves; ++hh)
                tma_load_3d(dst + hh * 16384, m, bar, hh * 64, rec.kstart, h);
              return;
            }
            const int rows = min(a.page_size, 128);
            for (int r0 = 0; r0 < 128; r0 += rows) {
              const int key = rec.kstart + r0;
              const int page = clamp_entry(a.block_table[min(key / a.page_size, a.table_len - 1)],
                                           0, a.num_pages - 1, p.status);
#pragma unroll
              for (int hh = 0; hh < C::kHalves; ++hh)
                tma_load_4d(dst + hh * 16384 + r0 * 128, m, bar, hh * 64, h, key % a.page_size,
                            page);
            }
          };
          good = mbar_wait(smem_u32(&k_empty[st]), par, wc);
          if (good) {
            load_tile(kst, mk, smem_u32(&k_full[st]), paged_k);
            good = mbar_wait(smem_u32(&v_empty[st]), par, wc);
          }
          if (good) load_tile(vst, mv, smem_u32(&v_full[st]), paged_v);
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) return false;
      } else {
        // Float32 pooled inputs: gather up to 64 listed entries in two parts --
        // rows e < 64 hold round(x), rows 64 + e hold round(x - round(x)) -- so
        // that Q.K^T accumulated over both parts carries the float32 pooled keys
        // and P.V over both parts the float32 pooled values.
        if (lane == 0) {
          good = mbar_wait(smem_u32(&k_empty[st]), par, wc);
          if (good) good = mbar_wait(smem_u32(&v_empty[st]), par, wc);
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) return false;
        constexpr int kChunks = D / 8;   // 16-byte chunks per tile row (past a.D: zeros)
        for (int idx = lane; idx < 128 * kChunks; idx += 32) {
          const int e = idx / kChunks, cidx = idx % kChunks;
          const int hh = cidx >> 3, cc = cidx & 7;
          const uint32_t off = hh * 16384 + e * 128 + ((cc ^ (e & 7)) << 4);
          const int ent = e & 63;
          const bool low = e >= 64;
          uint4 kvk = make_uint4(0, 0, 0, 0), kvv = make_uint4(0, 0, 0, 0);
          if (ent < rec.nvalid && cidx * 8 < a.D) {
            const int blk = clamp_entry(a.pr_ids[lrow + rec.kstart + ent], 0, a.Nb - 1, p.status);
            const long long src = ((long long)h * a.Nb + blk) * a.D + cidx * 8;
            const float4* fk = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.pk) + src);
            const float4* fv = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.pv) + src);
            const float4 k0 = __ldg(fk), k1 = __ldg(fk + 1), v0 = __ldg(fv), v1 = __ldg(fv + 1);
            kvk = make_uint4(pack2_split<DT>(k0.x, k0.y, low), pack2_split<DT>(k0.z, k0.w, low),
                             pack2_split<DT>(k1.x, k1.y, low), pack2_split<DT>(k1.z, k1.w, low));
            const float vs = a.v_exp != nullptr ? ldexpf(1.f, -a.v_exp[h]) : 1.f;
            kvv = make_uint4(pack2_split<VT>(v0.x * vs, v0.y * vs, low),
                             pack2_split<VT>(v0.z * vs, v0.w * vs, low),
                             pack2_split<VT>(v1.x * vs, v1.y * vs, low),
                             pack2_split<VT>(v1.z * vs, v1.w * vs, low));
          }
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(kst + off), "r"(kvk.x),
                       "r"(kvk.y), "r"(kvk.z), "r"(kvk.w)
                       : "memory");
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(vst + off), "r"(kvv.x),
                       "r"(kvv.y), "r"(kvv.z), "r"(kvv.w)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(&k_full[st]));
          mbar_arrive(smem_u32(&v_full[st]));
        }
      }
      ++kv;
      return true;
    };

    for (int w = next_work(); w < p.items && ok; w = next_work()) {
      const Pair pr = make_pair(p, w);
      const long long lrow = ((long long)pr.h * a.Nt + pr.t) * a.Nb;
      const int nsel = clamp_entry(a.sel_counts[(long long)pr.h * a.Nt + pr.t], 0, a.Nb, p.status);
      const int npr = a.corr ? clamp_entry(a.pr_counts[(long long)pr.h * a.Nt + pr.t], 0, a.Nb, p.status) : 0;
      // Selected blocks up to the first one past the chunks (fpv2/kernel.py:249-255).
      int n_sel_items = 0, brk = nsel;
      for (int i0 = 0; i0 < nsel; i0 += 32) {
        const int i = i0 + lane;
        const bool in = i < nsel;
        const int blk = in ? clamp_entry(a.sel_ids[lrow + i], 0, a.Nb - 1, p.status) : 0;
        const long long bstart = (long long)blk * a.block_k;
        const unsigned stop = __ballot_sync(0xffffffffu, in && bstart > pr.abs_last);
        const int lim = stop ? (__ffs(stop) - 1) : 32;
        int contrib = 0;
        if (in && lane < lim) contrib = (int)min((long long)bk_sub, (pr.abs_last - bstart) / 128 + 1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
        n_sel_items += contrib;
        if (stop) { brk = i0 + lim; break; }
      }
      // Pooled correction items.
      int n_corr_items = 0;
      const int n_ptiles = (a.Nb + 127) / 128;
      if (pool_tiles && npr > 0) {
        const int nwords = (a.Nb + 31) / 32;
        for (int i = lane; i < nwords; i += 32) pmask[i] = 0u;
        __syncwarp();
        for (int i = lane; i < npr; i += 32) {
          const int blk = clamp_entry(a.pr_ids[lrow + i], 0, a.Nb - 1, p.status);
          atomicOr(&pmask[blk >> 5], 1u << (blk & 31));
        }
        __syncwarp();
        for (int j = 0; j < n_ptiles; ++j) {
          const int w0 = 4 * j;
          uint32_t any = 0;
          for (int x = 0; x < 4 && w0 + x < nwords; ++x) any |= pmask[w0 + x];
          n_corr_items += any != 0u;
        }
      } else if (npr > 0) {
        n_corr_items = (npr + 63) / 64;   // 64 entries (high + low parts) per item
      }
      const int n_items = n_sel_items + n_corr_items;
      // Q tiles of both chunks (a work item without keys needs none).
      if (n_items > 0) {
        for (int x = 0; x < 2 && ok; ++x) {
          const int qs = qcount % kQSlots;
          if (lane == 0)
            ok = mbar_wait(smem_u32(&q_empty[qs]), ((qcount / kQSlots) & 1) ^ 1, wc);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (ok && lane == 0) {
            const uint32_t qb = smem_u32(&q_full[qs]);
            mbar_arrive_expect_tx(qb, (uint32_t)C::kTileBytes);
#pragma unroll
            for (int hh = 0; hh < C::kHalves; ++hh)
              tma_load_3d(q_smem + qs * C::kTileBytes + hh * 16384, &tmap_q, qb, hh * 64,
                          pr.t * a.tile_q + pr.p0, pr.h * a.G + pr.g0[x]);
          }
          ++qcount;
        }
        if (!ok) break;
      }
      int emitted = 0;
      auto make_rec = [&](int kind, int kstart, int nvalid) {
        Rec r;
        r.kind = kind;
        r.kstart = kstart;
        r.nvalid = nvalid;
        r.flags = (emitted == 0 ? 1 : 0) | (emitted == max(1, n_items) - 1 ? 2 : 0);
        r.w = w;
        r.part = -1;
        r.mask[0] = r.mask[1] = r.mask[2] = r.mask[3] = 0u;
        ++emitted;
        return r;
      };
      for (int i0 = 0; i0 < brk && ok; i0 += 32) {
        const int i = i0 + lane;
        const int blk = i < brk ? clamp_entry(a.sel_ids[lrow + i], 0, a.Nb - 1, p.status) : 0;
        const int cnt = min(32, brk - i0);
        for (int j = 0; j < cnt && ok; ++j) {
          const int bj = __shfl_sync(0xffffffffu, blk, j);
          const long long bstart = (long long)bj * a.block_k;
          for (int sub = 0; sub < bk_sub && ok; ++sub) {
            const long long ks = bstart + sub * 128;
            if (ks > pr.abs_last) break;
            ok = emit(make_rec(KIND_SEL, (int)ks, 0), pr.h, lrow);
          }
        }
      }
      if (pool_tiles) {
        const int nwords = (a.Nb + 31) / 32;
        for (int j = 0; j < n_ptiles && ok && npr > 0; ++j) {
          uint32_t m4[4];
          uint32_t any = 0;
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            m4[x] = (4 * j + x < nwords) ? pmask[4 * j + x] : 0u;
            any |= m4[x];
          }
          if (!any) continue;
          Rec r = make_rec(KIND_POOL, j * 128, 0);
#pragma unroll
          for (int x = 0; x < 4; ++x) r.mask[x] = m4[x];
          ok = emit(r, pr.h, lrow);
        }
        __syncwarp();   // pmask reads done before the next work item clears it
      } else {
        for (int j = 0; j < n_corr_items && ok; ++j)
          ok = emit(make_rec(KIND_CORR, j * 64, min(64, npr - j * 64)), pr.h, lrow);
      }
      if (ok && n_items == 0) ok = emit(make_rec(KIND_EMPTY, 0, 0), pr.h, lrow);
    }
    if (ok) {
      Rec done;
      done.kind = KIND_DONE;
      done.kstart = done.nvalid = done.w = 0;
      done.part = -1;
      done.flags = 3;
      done.mask[0] = done.mask[1] = done.mask[2] = done.mask[3] = 0u;
      emit(done, 0, 0);
    }
    // Drain in-flight bulk copies before the CTA retires.
    if (lane == 0) {
      for (int i = 0; i < kStages; ++i) {
        const int uses = (kv - i + kStages - 1) / kStages;
        if (uses > 0) {
          mbar_wait(smem_u32(&k_full[i]), (uses - 1) & 1, wc, false);
          mbar_wait(smem_u32(&v_full[i]), (uses - 1) & 1, wc, false);
        }
      }
      for (int i = 0; i < kQSlots; ++i) {
        const int uses = (qcount - i + kQSlots - 1) / kQSlots;
        if (uses > 0) mbar_wait(smem_u32(&q_full[i]), (uses - 1) & 1, wc, false);
      }
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ==============================
    if (lane == 0) {
      int qcount = 0, icount = 0, kv = 0;
      int qs[2] = {0, 0};
      bool ok = true;
      int pb = -1;                 // kv index whose PV_B is pending
      bool pb_first = false, pb_last = false, pb_corr = false;
      auto issue_qk = [&](int x, int st, bool corr) {
        const uint32_t s_tmem = tmem_base + C::kSCol + x * 128;
        const uint32_t qb = q_smem + qs[x] * C::kTileBytes;
        const uint32_t kb = k_smem + st * C::kTileBytes;
        if (!corr) {
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int hh = kk / 4, sub = kk % 4;
            const uint64_t adesc = sw128_desc(qb + hh * 16384 + sub * 32, 16, 1024);
            const uint64_t bdesc = sw128_desc(kb + hh * 16384 + sub * 32, 16, 1024);
            umma_ss(s_tmem, adesc, bdesc, p.idesc_qk, kk > 0 ? 1u : 0u);
          }
        } else {
          // gathered CORR item: S[:, 0:64] = Q.K_high^T + Q.K_low^T (key rows 0..63
          // and 64..127, 8 KB apart in each 64-column box), N = 64, one accumulator
#pragma unroll
          for (int part = 0; part < 2; ++part) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int hh = kk / 4, sub = kk % 4;
              const uint64_t adesc = sw128_desc(qb + hh * 16384 + sub * 32, 16, 1024);
              const uint64_t bdesc = sw128_desc(kb + hh * 16384 + part * 8192 + sub * 32, 16, 1024);
              umma_ss(s_tmem, adesc, bdesc, p.idesc_qk64, (part | kk) ? 1u : 0u);
            }
          }
        }
        umma_commit(smem_u32(&s_full[x]));
      };
      // O_x += P_x V, each 64-key half as soon as its four softmax warps are done;
      // P (128 keys, 16-bit pairs) sits in the first 64 of the S columns.
      auto issue_pv = [&](int x, int n, bool first, bool last, bool corr) -> bool {
        const int st = n % kStages;
        const uint32_t par = (n / kStages) & 1;
        if (!mbar_wait(smem_u32(&v_full[st]), par, wc)) return false;
        const uint32_t s_tmem = tmem_base + C::kSCol + x * 128;
        const uint32_t vst = v_smem + st * C::kTileBytes;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(smem_u32(&p_full[2 * x + h]), n & 1, wc)) return false;
          tc_fence_after();
          // (CORR: P of the 64 entries times the high value rows 0..63, then the
          // same P times the low value rows 64..127)
          const uint32_t pcol = corr ? 0u : 32u * h;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bdesc = sw128_desc(vst + (4 * h + kk) * 2048, 16384, 1024);
            umma_ts(tmem_base + C::kOCol + x * 128, s_tmem + pcol + kk * 8, bdesc, p.idesc_pv,
                    (first && h == 0 && kk == 0) ? 0u : 1u);
          }
        }
        umma_commit(smem_u32(&pv_done[x]));
        if (x == 1) umma_commit(smem_u32(&v_empty[st]));   // PV_A of this tile went first
        if (last) umma_commit(smem_u32(&o_full[x]));
        return true;
      };
      while (ok) {
        const int ri = icount % kRecs;
        ok = mbar_wait(smem_u32(&rec_full[ri]), (icount / kRecs) & 1, wc);
        if (!ok) break;
        const Rec rec = recs[ri];
        mbar_arrive(smem_u32(&rec_empty[ri]));
        ++icount;
        if (rec.kind == KIND_DONE) break;
        if (rec.kind == KIND_EMPTY) continue;
        const bool first = rec.flags & 1, last = (rec.flags & 2) != 0;
        const int st = kv % kStages;
        const uint32_t par = (kv / kStages) & 1;
        ok = mbar_wait(smem_u32(&k_full[st]), par, wc);
        if (!ok) break;
        if (first) {
          qs[0] = qcount % kQSlots;
          qs[1] = (qcount + 1) % kQSlots;
          ok = mbar_wait(smem_u32(&q_full[qs[0]]), (qcount / kQSlots) & 1, wc);
          if (ok) ok = mbar_wait(smem_u32(&q_full[qs[1]]), ((qcount + 1) / kQSlots) & 1, wc);
          if (!ok) break;
          qcount += 2;
        }
        tc_fence_after();
        const bool corr = rec.kind == KIND_CORR;
        issue_qk(0, st, corr);
        if (last) umma_commit(smem_u32(&q_empty[qs[0]]));
        if (pb >= 0) {
          ok = issue_pv(1, pb, pb_first, pb_last, pb_corr);
          if (!ok) break;
          pb = -1;
        }
        issue_qk(1, st, corr);
        umma_commit(smem_u32(&k_empty[st]));
        if (last) umma_commit(smem_u32(&q_empty[qs[1]]));
        ok = issue_pv(0, kv, first, last, corr);
        if (!ok) break;
        pb = kv;
        pb_first = first;
        pb_last = last;
        pb_corr = corr;
        ++kv;
      }
      if (ok && pb >= 0) issue_pv(1, pb, pb_first, pb_last, pb_corr);
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, wc, false);
    }
  }
  } else {
    regs_inc<kRegsHigh>();
    // ======================= softmax + output ==============================
    const int x = (warp - 4) >> 2;              // 0: chunk A, 1: chunk B
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;          // row of the 128-row chunk
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_tmem = tmem_base + lane_off + C::kOCol + x * 128;
    const uint32_t s_tmem = tmem_base + lane_off + C::kSCol + x * 128;
    const float c2 = a.scale_log2;
    int icount = 0, kv = 0, nfull = 0;
    bool ok = true;
    long long row = 0, position = 0, head = 0;
    int kvh = 0;
    bool row_valid = false;
    float m_used = kFiniteMin, l = 0.f;
    int pv_cnt = 0;
    while (ok) {
      const int ri = icount % kRecs;
      ok = mbar_wait(smem_u32(&rec_full[ri]), (icount / kRecs) & 1, wc);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const Rec rec = recs[ri];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&rec_empty[ri]));
      ++icount;
      if (rec.kind == KIND_DONE) break;
      if (rec.flags & 1) {
        const Pair pr = make_pair(p, rec.w);
        kvh = pr.h;
        const int P = pr.c[x] * 128 + r;
        row = (long long)pr.t * a.tile_q + P % a.tile_q;
        head = (long long)pr.h * a.G + P / a.tile_q;
        position = (long long)a.offset + row;
        row_valid = row < a.valid_lq;
        m_used = kFiniteMin;
        l = 0.f;
        pv_cnt = 0;
      }
      if (rec.kind != KIND_EMPTY) {
        ok = mbar_wait(smem_u32(&s_full[x]), kv & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        uint32_t s[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + 32 * c, s[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) reg_fence(s[c]);
        // validity of the 128 entries; a warp with any invalid entry masks on every lane
        float bias = 0.f;
        uint32_t vm[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
        bool full = true;
        if (rec.kind == KIND_SEL) {
          const long long ks = rec.kstart;
          const bool row_full = row_valid && ks + 127 <= position && ks + 127 < a.valid_lk;
          full = __all_sync(0xffffffffu, row_full);
          if (!full) {
            const long long lim = row_valid ? min(position + 1, (long long)a.valid_lk) - ks : 0;
#pragma unroll
            for (int c = 0; c < 4; ++c) vm[c] = prefix_mask(lim - 32 * c);
          }
        } else if (rec.kind == KIND_POOL) {
          bias = a.corr_shift;
          full = false;
#pragma unroll
          for (int c = 0; c < 4; ++c) vm[c] = rec.mask[c];
        } else {   // KIND_CORR (at most 64 entries)
          bias = a.corr_shift;
          full = rec.nvalid >= 128;
          if (!full) {
#pragma unroll
            for (int c = 0; c < 4; ++c) vm[c] = prefix_mask(rec.nvalid - 32 * c);
          }
        }
        // Full warps keep the raw scores (c2 > 0 keeps the order; x = s*c2 + bias
        // is formed inside the exponent); otherwise x = s*c2 + bias with masked
        // entries at finite_min, exactly as the reference kernel masks its logits.
        if (!full) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float xv = fmaf(__uint_as_float(s[c][j]), c2, bias);
              s[c][j] = ((vm[c] >> j) & 1u) ? __float_as_uint(xv) : __float_as_uint(kFiniteMin);
            }
          }
        }
        float mt;
        {
          float mx[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            mx[c] = max3f(__uint_as_float(s[c][0]), __uint_as_float(s[c][1]), __uint_as_float(s[c][2]));
#pragma unroll
            for (int j = 3; j < 31; j += 2)
              mx[c] = max3f(mx[c], __uint_as_float(s[c][j]), __uint_as_float(s[c][j + 1]));
            mx[c] = fmaxf(mx[c], __uint_as_float(s[c][31]));
          }
          const float m4 = max3f(mx[0], mx[1], fmaxf(mx[2], mx[3]));
          mt = full ? fmaf(m4, c2, bias) : m4;
        }
        const float m_new = fmaxf(m_used, mt);
        const bool need = m_new > m_used + RescaleT<VT>::value ||
                          (m_used == kFiniteMin && m_new > kFiniteMin);
        if (__any_sync(0xffffffffu, need)) {
          const float f = need ? ex2(m_used - m_new) : 1.f;
          if (need) {
            m_used = m_new;
            l *= f;
          }
          if (pv_cnt > 0) {
            // O holds PVs of this work item: wait for the latest one, rescale.
            ok = mbar_wait(smem_u32(&pv_done[x]), (kv - 1) & 1, wc);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
#pragma unroll 1
            for (int dc = 0; dc < D / 32; ++dc) {
              uint32_t o[32];
              tmem_ld32(o_tmem + dc * 32, o);
              tmem_wait_ld();
              reg_fence(o);
#pragma unroll
              for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f);
              tmem_st32(o_tmem + dc * 32, o);
            }
            tmem_wait_st();
          }
        }
        // P = 2^(x - m): a masked entry (x = finite_min) weighs 1 while the row has
        // seen nothing but masked entries (m = finite_min), else 0.
        const float2 cm2 = full ? make_float2(c2, c2) : make_float2(1.f, 1.f);
        const float2 nb2 = full ? make_float2(bias - m_used, bias - m_used) : make_float2(-m_used, -m_used);
        float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t pk[32];
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              const int c = 2 * h + cc;
              const float2 xv = fma_f32x2(
                  make_float2(__uint_as_float(s[c][2 * q]), __uint_as_float(s[c][2 * q + 1])), cm2, nb2);
              float2 pv;
              pv.x = ex2(xv.x);
              pv.y = ex2(xv.y);
              rs[q & 3] = add_f32x2(rs[q & 3], pv);
              pk[16 * cc + q] = pack_p<VT>(pv.x, pv.y);
            }
          }
          // P of keys 64h .. 64h+63 -> S columns 32h .. 32h+31 (already read)
          tmem_st32(s_tmem + 32 * h, pk);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&p_full[2 * x + h]));
        }
        l += ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y));
        ++kv;
        ++pv_cnt;
      }
      if (rec.flags & 2) {
        // ---- output row: O / l, written straight from registers
        // (times 2^v_exp[h] when V was scaled into the fp16 range)
        const float vsc = a.v_exp != nullptr ? ldexpf(1.f, a.v_exp[kvh]) : 1.f;
        const float inv = (pv_cnt > 0 && l > 0.f) ? vsc / l : 0.f;
        if (pv_cnt > 0) {
          ok = mbar_wait(smem_u32(&o_full[x]), nfull & 1, wc);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          ++nfull;
          tc_fence_after();
        }
        char* dst_row = reinterpret_cast<char*>(a.out) + (head * a.Lq_pad + row) * a.D * 2;
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          if (dc * 32 >= a.D) break;   // head_dim 96 runs on the 128-wide tiles
          uint32_t o[32];
          if (pv_cnt > 0) {
            tmem_ld32(o_tmem + dc * 32, o);
            tmem_wait_ld();
            reg_fence(o);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = 0u;
          }
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 v;
            v.x = pack2<DT>(__uint_as_float(o[8 * j + 0]) * inv, __uint_as_float(o[8 * j + 1]) * inv);
            v.y = pack2<DT>(__uint_as_float(o[8 * j + 2]) * inv, __uint_as_float(o[8 * j + 3]) * inv);
            v.z = pack2<DT>(__uint_as_float(o[8 * j + 4]) * inv, __uint_as_float(o[8 * j + 5]) * inv);
            v.w = pack2<DT>(__uint_as_float(o[8 * j + 6]) * inv, __uint_as_float(o[8 * j + 7]) * inv);
            char* dst = dst_row + (dc * 32 + 8 * j) * 2;
            *reinterpret_cast<uint4*>(dst) = v;
          }
        }
        tc_fence_before();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

template <int D>
size_t pair_smem_bytes() {
  return 1024 + (size_t)(kQSlots + 2 * kStages) * PCfg<D>::kTileBytes + sizeof(Rec) * kRecs +
         4 * kMaskWordsMax + 8 * (2 * kQSlots + 2 * kRecs + 4 * kStages + 11) + 16;
}

}  // namespace

bool attn_pair_supported(const AttnArgs& a) {
  if (!attn_tc_supported(a)) return false;
  if (a.out_mc != nullptr) return false;   // multicast output stays on attn_tc_kernel
  const int nch = (a.G * a.tile_q) / 128;
  const int cpg = a.tile_q >= 128 ? a.tile_q / 128 : 1;
  return nch >= 2 && (nch / cpg) % 2 == 0;
}

cudaError_t launch_attn_pair(const AttnArgs& a, const TcLaunch& L, int* sched, cudaStream_t stream) {
  Params p;
  p.a = a;
  p.nch = (a.G * a.tile_q) / 128;
  p.items = a.Hkv * a.Nt * (p.nch / 2);
  const int fmt = a.dt == DT_BF16 ? 1 : 0;
  const int vdt = a.vdt < 0 ? a.dt : a.vdt;
  p.idesc_qk = umma_idesc_f16(fmt, 128, 128, 0, 0);
  p.idesc_qk64 = umma_idesc_f16(fmt, 128, 64, 0, 0);
  p.idesc_pv = umma_idesc_f16(vdt == DT_BF16 ? 1 : 0, 128, a.D, 0, 1);
  p.sched = sched;
  p.status = L.status;
  p.budget = L.budget;
  if (p.items == 0) return cudaSuccess;
  CUtensorMap m[6];
  if (!encode_attn_maps(a, m)) return cudaErrorInvalidValue;
  const int grid = max(1, min(L.num_sms, p.items));
  cudaError_t e = cudaSuccess;
  if (sched != nullptr) {
    e = cudaMemsetAsync(sched, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
#define FPV2_PAIR_LAUNCH(DD, TT, VV)                                                        \
  {                                                                                         \
    const size_t smem = pair_smem_bytes<DD>();                                              \
    e = cudaFuncSetAttribute(attn_pair_kernel<DD, TT, VV>,                                  \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);       \
    if (e != cudaSuccess) return e;                                                         \
    attn_pair_kernel<DD, TT, VV><<<grid, kThreads, smem, stream>>>(m[0], m[1], m[2], m[3], m[4], p); \
    count_launch();                                                                         \
  }
  if (a.D == 64 && a.dt == DT_BF16 && vdt == DT_F16) FPV2_PAIR_LAUNCH(64, DT_BF16, DT_F16)
  else if (a.D == 64 && a.dt == DT_BF16) FPV2_PAIR_LAUNCH(64, DT_BF16, DT_BF16)
  else if (a.D == 64 && a.dt == DT_F16) FPV2_PAIR_LAUNCH(64, DT_F16, DT_F16)
  // head_dim 96 runs on the 128-wide tiles (TMA zero-fills columns 96..127,
  // PV runs with N = 96, output rows stop at column 96)
  else if (a.D >= 96 && a.dt == DT_BF16 && vdt == DT_F16) FPV2_PAIR_LAUNCH(128, DT_BF16, DT_F16)
  else if (a.D >= 96 && a.dt == DT_BF16) FPV2_PAIR_LAUNCH(128, DT_BF16, DT_BF16)
  else if (a.D >= 96 && a.dt == DT_F16) FPV2_PAIR_LAUNCH(128, DT_F16, DT_F16)
  else return cudaErrorInvalidValue;
#undef FPV2_PAIR_LAUNCH
  return cudaGetLastError();
}

}  // namespace fpv2
