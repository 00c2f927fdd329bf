// Block-sparse attention on tensor cores (tcgen05 + TMEM + TMA).
//
// Math (fpv2/kernel.py:187-414): for each query row, an online softmax in
// base 2 over the keys of the selected blocks (causal / key_length masked,
// masked logits = finite_min), followed by the pruned blocks as pooled K/V
// entries whose logits are shifted by log2(block_k); out = O / l.
//
// A work item is one 128-row chunk of a selection tile: the G query heads of
// one KV head packed together (GQA packing), so every K/V tile loaded feeds
// all G heads. Per KV item (one 128-key sub-tile of a selected block, or one
// 128-row tile of pooled K/V):
//   S[128x128] = Q . K^T          tcgen05.mma SS, fp32 in TMEM (double buffered)
//   P = 2^(S*c - m)               softmax warps: TMEM -> regs -> bf16/f16 P back
//                                 into the same TMEM columns
//   O_h[128xD] += P_h . V_h       tcgen05.mma TS (A = P from TMEM, B = V MN-major)
// Each 128-key S tile is split into two 64-key halves h with fully separate
// online-softmax state: a half has its own running max m_h, sum l_h and
// accumulator O_h in TMEM (TMEM = O_0 | O_1 | S buffer 0 | S buffer 1, 4 x 128
// columns). The two halves of a row are combined once per work item:
//   out = (2^(m_0-m) O_0 + 2^(m_1-m) O_1) / (2^(m_0-m) l_0 + 2^(m_1-m) l_1),
// m = max(m_0, m_1), which equals the single online softmax over all keys.
// So the two warps that share a row never exchange anything per KV item.
// Each running max is rescaled lazily: O_h is only rescaled when m_h grows by
// more than a factor 2^16 (2^15 for fp16), which leaves the final result
// unchanged. The softmax arithmetic runs on packed fp32 pairs (one FMA and one
// add per two keys) and three-input maxima, which leaves the MUFU exponentials
// as the only per-key scalar work.
//
// Pooled correction: instead of gathering the pruned blocks' pooled rows, the
// producer streams contiguous 128-row tiles of the head's pooled K/V with TMA
// and ships a 128-bit mask per tile (bit = "this pooled entry is in the pruned
// list"); masked entries take finite_min logits, exactly like list padding in
// the reference kernel. Tiles without a pruned entry are skipped. Pooled
// inputs in float32 (the semantics of fpv2/reference.py) take a gathered path
// that keeps their precision: each CORR item holds up to 64 pruned entries,
// key/value rows 0..63 the 16-bit high parts and rows 64..127 the low parts
// (x - high). The issuer accumulates Q.K_high^T + Q.K_low^T into the same 64
// score columns (two N = 64 chains) and P.V_high + P.V_low into O_0, so the
// softmax sees an ordinary 64-entry item (its second half fully masked).
//
// Warp roles (320 threads, one persistent CTA per SM):
//   warp 0     producer: takes work items from a global counter (largest
//              first), walks the lists, publishes one record per KV item and
//              loads Q / K / V / pooled tiles with TMA (no multicast);
//   warp 1     MMA issuer;
//   warps 2-9  softmax and the output epilogue: two warps per TMEM lane
//              quarter (thread = query row), each owning one 64-key half of
//              every S tile and its accumulator O_h; in the epilogue each
//              writes half of the output columns.
#include "attn_common.cuh"

#include <algorithm>

namespace fpv2 {

namespace {

constexpr int kThreads = 320;   // producer, MMA, 8 softmax warps
constexpr int kStages = 2;      // K/V tiles and S buffers
constexpr int kRecs = 8;        // item records in flight
constexpr int kTmemCols = 512;
template <int D>
struct Cfg {
  static constexpr int kHalves = D / 64;
  static constexpr int kTileBytes = 128 * D * 2;   // Q, K or V tile
  static constexpr int kOCol = 0;                  // O_h at columns [128 h, 128 h + D)
  static constexpr int kSCol = 256;                // S buffers at 256, 384
};

// DT: input dtype; VT: operand type of the P.V product (V and P); GATHER: the
// pooled correction is gathered from float32 pooled K/V (CORR items) instead of
// streamed as pooled tiles (compiled out of the other instantiations).
template <int D, int DT, int VT, bool GATHER>
__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                   const __grid_constant__ CUtensorMap tmap_k,
                   const __grid_constant__ CUtensorMap tmap_v,
                   const __grid_constant__ CUtensorMap tmap_pk,
                   const __grid_constant__ CUtensorMap tmap_pv,
                   const __grid_constant__ CUtensorMap tmap_o, Params p) {
  using C = Cfg<D>;
  const AttnArgs& a = p.a;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);

  const uint32_t q_smem = base;                                   // [2][tile]
  const uint32_t k_smem = base + 2 * C::kTileBytes;               // [kStages][tile]
  const uint32_t v_smem = k_smem + kStages * C::kTileBytes;       // [kStages][tile]
  uint8_t* after_tiles = gbase + (2 + 2 * kStages) * C::kTileBytes;
  Rec* recs = reinterpret_cast<Rec*>(after_tiles);                // [kRecs]
  uint32_t* pmask = reinterpret_cast<uint32_t*>(recs + kRecs);    // producer-private [64]
  float* xm = reinterpret_cast<float*>(pmask + kMaskWordsMax);    // [2 parity][2 half][128] m_h
  float* lsum = xm + 2 * 2 * 128;                                  // [2 parity][2 half][128] l_h
  uint64_t* bars = reinterpret_cast<uint64_t*>(lsum + 2 * 2 * 128);
  uint64_t* q_full = bars;              // [2]
  uint64_t* q_empty = q_full + 2;       // [2]
  uint64_t* rec_full = q_empty + 2;     // [kRecs]
  uint64_t* rec_empty = rec_full + kRecs;
  uint64_t* k_full = rec_empty + kRecs; // [kStages]
  uint64_t* k_empty = k_full + kStages;
  uint64_t* v_full = k_empty + kStages;
  uint64_t* v_empty = v_full + kStages;
  uint64_t* s_full = v_empty + kStages;
  uint64_t* p_full = s_full + kStages;  // [kStages][2 half] (4 warps each)
  uint64_t* pv_done = p_full + 2 * kStages;  // [1]
  uint64_t* o_full = pv_done + 1;        // [1]
  uint64_t* o_free = o_full + 1;         // [1]
  uint64_t* drain = o_free + 1;          // [1]
  uint64_t* lbar = drain + 1;            // [4] epilogue (m_h, l_h) exchange of a warp pair
  uint64_t* obar = lbar + 4;             // [2] output tile staged (per 64-column box)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(obar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&q_full[i]), 1);
      // last QK + the output stores (two tensor stores, or eight warps' multicast stores)
      mbar_init(smem_u32(&q_empty[i]), 1 + (a.out_mc != nullptr ? 8 : 2));
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
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[2 * i]), 4);
      mbar_init(smem_u32(&p_full[2 * i + 1]), 4);
    }
    mbar_init(smem_u32(pv_done), 1);
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(o_free), 8);
    mbar_init(smem_u32(drain), 1);
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&lbar[i]), 2);
    mbar_init(smem_u32(&obar[0]), D == 128 ? 4 : 8);
    mbar_init(smem_u32(&obar[1]), 4);
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
  const bool pool_tiles = a.corr && !GATHER;   // TMA pooled tiles vs gather

  if (warp == 0) {
    // ============================ producer ================================
    int qcount = 0, icount = 0, kv = 0, wstatic = blockIdx.x;
    bool ok = true;
    const bool split = p.split.max_slots > 0 && p.sched != nullptr;
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
    // Units: kMaxSeg per item of the first max_slots items (w, s), then the other
    // items one each (s = -1).
    const int n_split_units = split ? p.split.max_slots * kMaxSeg : 0;
    const int n_units = split ? n_split_units + p.items - p.split.max_slots : p.items;
    // Publish one record; SEL/POOL/CORR records are followed by their K/V tiles.
    auto emit = [&](const Rec& rec, const Chunk& ck, long long lrow) -> bool {
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
          // One 128-row tile: a single 3-D box per 64 features, or, from a page
          // pool, one 4-D box per page the 128 keys span.
          auto load_tile = [&](uint32_t dst, const CUtensorMap* m, uint32_t bar, bool paged) {
            mbar_arrive_expect_tx(bar, (uint32_t)C::kTileBytes);
            if (!paged) {
#pragma unroll
              for (int hh = 0; hh < C::kHalves; ++hh)
                tma_load_3d(dst + hh * 16384, m, bar, hh * 64, rec.kstart, ck.h);
              return;
            }
            const int rows = min(a.page_size, 128);
            for (int r0 = 0; r0 < 128; r0 += rows) {
              const int key = rec.kstart + r0;
              const int page = clamp_entry(a.block_table[min(key / a.page_size, a.table_len - 1)],
                                           0, a.num_pages - 1, p.status);
#pragma unroll
              for (int hh = 0; hh < C::kHalves; ++hh)
                tma_load_4d(dst + hh * 16384 + r0 * 128, m, bar, hh * 64, ck.h, key % a.page_size,
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
            const long long src = ((long long)ck.h * a.Nb + blk) * a.D + cidx * 8;
            const float4* fk = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.pk) + src);
            const float4* fv = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(a.pv) + src);
            const float4 k0 = __ldg(fk), k1 = __ldg(fk + 1), v0 = __ldg(fv), v1 = __ldg(fv + 1);
            kvk = make_uint4(pack2_split<DT>(k0.x, k0.y, low), pack2_split<DT>(k0.z, k0.w, low),
                             pack2_split<DT>(k1.x, k1.y, low), pack2_split<DT>(k1.z, k1.w, low));
            const float vs = a.v_exp != nullptr ? ldexpf(1.f, -a.v_exp[ck.h]) : 1.f;
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

    for (int u = next_work(); u < n_units && ok; u = next_work()) {
      const bool vunit = u < n_split_units;
      const int w = vunit ? u / kMaxSeg : u - n_split_units + p.split.max_slots;
      const int seg = vunit ? u % kMaxSeg : -1;
      const Chunk ck = make_chunk(p, w);
      const long long lrow = ((long long)ck.h * a.Nt + ck.t) * a.Nb;
      const int nsel = clamp_entry(a.sel_counts[(long long)ck.h * a.Nt + ck.t], 0, a.Nb, p.status);
      const int npr = a.corr ? clamp_entry(a.pr_counts[(long long)ck.h * a.Nt + ck.t], 0, a.Nb, p.status) : 0;
      // Q tile of the chunk (a split unit loads it once it knows it runs).
      auto load_q = [&]() -> bool {
        const int qs = qcount & 1;
        bool good = true;
        if (lane == 0) good = mbar_wait(smem_u32(&q_empty[qs]), ((qcount >> 1) & 1) ^ 1, wc);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) return false;
        if (lane == 0) {
          const uint32_t qb = smem_u32(&q_full[qs]);
          mbar_arrive_expect_tx(qb, (uint32_t)C::kTileBytes);
#pragma unroll
          for (int hh = 0; hh < C::kHalves; ++hh)
            tma_load_3d(q_smem + qs * C::kTileBytes + hh * 16384, &tmap_q, qb, hh * 64,
                        ck.t * a.tile_q + ck.p0, ck.h * a.G + ck.g0);
        }
        ++qcount;
        return true;
      };
      if (!vunit) {
        ok = load_q();
        if (!ok) break;
      }
      // A split unit first bounds the item's KV item count from its counts alone
      // (every listed block once, every pooled tile or 64 gathered entries once)
      // and skips at once when the item needs no segment s.
      int nseg = 1;
      if (vunit) {
        const int ub = nsel * bk_sub +
                       (a.corr ? (pool_tiles ? min(npr, (a.Nb + 127) / 128) : (npr + 63) / 64) : 0);
        if (ub > 2 * kSegLen) nseg = min(kMaxSeg, (ub + kSegLen - 1) / kSegLen);
        if (seg >= nseg) continue;   // a unit this item does not need
      }
      // Selected blocks up to the first one past the chunk (fpv2/kernel.py:249-255),
      // four independent 32-entry loads in flight per step.
      int n_sel_items = 0, brk = nsel;
      for (int i0 = 0; i0 < nsel; i0 += 128) {
        int blk4[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int i = i0 + 32 * x + lane;
          blk4[x] = i < nsel ? clamp_entry(a.sel_ids[lrow + i], 0, a.Nb - 1, p.status) : 0;
        }
        bool stopped = false;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int c0 = i0 + 32 * x;
          if (c0 >= nsel) break;
          const bool in = c0 + lane < nsel;
          const long long bstart = (long long)blk4[x] * a.block_k;
          const unsigned stop = __ballot_sync(0xffffffffu, in && bstart > ck.abs_last);
          const int lim = stop ? (__ffs(stop) - 1) : 32;
          int contrib = 0;
          if (in && lane < lim) contrib = (int)min((long long)bk_sub, (ck.abs_last - bstart) / 128 + 1);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) contrib += __shfl_xor_sync(0xffffffffu, contrib, o);
          n_sel_items += contrib;
          if (stop) {
            brk = c0 + lim;
            stopped = true;
            break;
          }
        }
        if (stopped) break;
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
      const int n_total = n_sel_items + n_corr_items;
      // This unit's share [lo, hi) of the item's KV item sequence.
      // (segments are equal shares of the exact count; the bound only sets nseg)
      int lo = 0, hi = n_total, part = -1;
      if (vunit) {
        if (nseg > 1) {
          const int per = (n_total + nseg - 1) / nseg;
          lo = min(n_total, seg * per);
          hi = seg == nseg - 1 ? n_total : min(n_total, lo + per);
          part = w * kMaxSeg + seg;
          if (seg == 0 && lane == 0) p.split.recs[w] = make_int4(w, nseg, 0, 0);
        }
        ok = load_q();
        if (!ok) break;
      }
      const int n_items = max(1, hi - lo);
      int emitted = 0, kvi = 0;   // kvi: index in the item's KV item sequence
      // With one 128-key item per listed block, the items before the first block
      // past the chunk are the blocks themselves: start at lo's 32-entry chunk.
      const int sel_start = bk_sub == 1 ? min(lo, brk) / 32 * 32 : 0;
      kvi = sel_start;
      auto make_rec = [&](int kind, int kstart, int nvalid) {
        Rec r;
        r.kind = kind;
        r.kstart = kstart;
        r.nvalid = nvalid;
        r.flags = (emitted == 0 ? 1 : 0) | (emitted == n_items - 1 ? 2 : 0);
        r.w = w;
        r.part = part;
        r.mask[0] = r.mask[1] = r.mask[2] = r.mask[3] = 0u;
        ++emitted;
        return r;
      };
      for (int i0 = sel_start; i0 < brk && ok && kvi < hi; i0 += 32) {
        const int i = i0 + lane;
        const int blk = i < brk ? clamp_entry(a.sel_ids[lrow + i], 0, a.Nb - 1, p.status) : 0;
        const int cnt = min(32, brk - i0);
        for (int j = 0; j < cnt && ok && kvi < hi; ++j) {
          const int bj = __shfl_sync(0xffffffffu, blk, j);
          const long long bstart = (long long)bj * a.block_k;
          for (int sub = 0; sub < bk_sub && ok && kvi < hi; ++sub) {
            const long long ks = bstart + sub * 128;
            if (ks > ck.abs_last) break;
            if (kvi++ < lo) continue;
            ok = emit(make_rec(KIND_SEL, (int)ks, 0), ck, lrow);
          }
        }
      }
      if (pool_tiles) {
        const int nwords = (a.Nb + 31) / 32;
        for (int j = 0; j < n_ptiles && ok && npr > 0 && kvi < hi; ++j) {
          uint32_t m4[4];
          uint32_t any = 0;
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            m4[x] = (4 * j + x < nwords) ? pmask[4 * j + x] : 0u;
            any |= m4[x];
          }
          if (!any) continue;
          if (kvi++ < lo) continue;
          Rec r = make_rec(KIND_POOL, j * 128, 0);
#pragma unroll
          for (int x = 0; x < 4; ++x) r.mask[x] = m4[x];
          ok = emit(r, ck, lrow);
        }
        __syncwarp();   // pmask reads done before the next work item clears it
      } else {
        for (int j = 0; j < n_corr_items && ok && kvi < hi; ++j) {
          if (kvi++ < lo) continue;
          ok = emit(make_rec(KIND_CORR, j * 64, min(64, npr - j * 64)), ck, lrow);
        }
      }
      if (ok && emitted == 0) ok = emit(make_rec(KIND_EMPTY, 0, 0), ck, lrow);
    }
    if (ok) {
      Rec done;
      done.kind = KIND_DONE;
      done.kstart = done.nvalid = done.w = 0;
      done.part = -1;
      done.flags = 3;
      done.mask[0] = done.mask[1] = done.mask[2] = done.mask[3] = 0u;
      Chunk none{};
      emit(done, none, 0);
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
      for (int i = 0; i < 2; ++i) {
        const int uses = (qcount - i + 1) / 2;
        if (uses > 0) mbar_wait(smem_u32(&q_full[i]), (uses - 1) & 1, wc, false);
      }
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ==============================
    if (lane == 0) {
      int qcount = 0, icount = 0, kv = 0, wi = 0, qs = 0;
      bool ok = true, need_ofree = false, first_pv = true;
      int prev = -1;   // kv index whose PV is pending
      bool prev_corr = false;   // that item is a gathered CORR item (high + low parts)
      auto issue_pv = [&](int n, bool corr) -> bool {
        const int st = n % kStages;
        const uint32_t par = (n / kStages) & 1;
        if (!mbar_wait(smem_u32(&v_full[st]), par, wc)) return false;
        if (need_ofree) {
          if (!mbar_wait(smem_u32(o_free), (wi - 1) & 1, wc)) return false;
          need_ofree = false;
        }
        const uint32_t s_tmem = tmem_base + C::kSCol + st * 128;
        const uint32_t vst = v_smem + st * C::kTileBytes;
        // O_h += P_h V_h, each half as soon as its four softmax warps are done;
        // P_h (64 keys, 16-bit pairs) sits in the first 32 of its S columns.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(smem_u32(&p_full[2 * st + h]), par, wc)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bdesc = sw128_desc(vst + (4 * h + kk) * 2048, 16384, 1024);
            umma_ts(tmem_base + C::kOCol + h * 128, s_tmem + 64 * h + kk * 8, bdesc, p.idesc_pv,
                    (first_pv && kk == 0) ? 0u : 1u);
          }
          if (corr && h == 0) {
            // CORR: the same P_0 times the low parts of the pooled values (rows 64..127)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t bdesc = sw128_desc(vst + (4 + kk) * 2048, 16384, 1024);
              umma_ts(tmem_base + C::kOCol, s_tmem + kk * 8, bdesc, p.idesc_pv, 1u);
            }
          }
        }
        first_pv = false;
        umma_commit(smem_u32(&v_empty[st]));
        umma_commit(smem_u32(pv_done));
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
        if (rec.flags & 1) {   // first item of a work item
          qs = qcount & 1;
          ok = mbar_wait(smem_u32(&q_full[qs]), (qcount >> 1) & 1, wc);
          if (!ok) break;
          ++qcount;
          need_ofree = wi > 0;
          first_pv = true;
          prev = -1;
        }
        if (rec.kind != KIND_EMPTY) {
          const int st = kv % kStages;
          const uint32_t par = (kv / kStages) & 1;
          // S buffer st held P of item kv - 2, read by a PV issued earlier from
          // this thread: tcgen05.mma ops run in issue order, so no wait here.
          ok = mbar_wait(smem_u32(&k_full[st]), par, wc);
          if (!ok) break;
          tc_fence_after();
          const uint32_t s_tmem = tmem_base + C::kSCol + st * 128;
          const uint32_t qb = q_smem + qs * C::kTileBytes;
          const uint32_t kb = k_smem + st * C::kTileBytes;
          const bool corr = GATHER && rec.kind == KIND_CORR;
          if (!corr) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int hh = kk / 4, sub = kk % 4;
              const uint64_t adesc = sw128_desc(qb + hh * 16384 + sub * 32, 16, 1024);
              const uint64_t bdesc = sw128_desc(kb + hh * 16384 + sub * 32, 16, 1024);
              umma_ss(s_tmem, adesc, bdesc, p.idesc_qk, kk > 0 ? 1u : 0u);
            }
          } else {
            // S[:, 0:64] = Q.K_high^T + Q.K_low^T: key rows 0..63 and 64..127 of the
            // gathered tile (8 KB apart in each 64-column box), N = 64, one accumulator
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
          umma_commit(smem_u32(&s_full[st]));
          umma_commit(smem_u32(&k_empty[st]));
          if (prev >= 0) ok = issue_pv(prev, prev_corr);
          if (!ok) break;
          prev = kv;
          prev_corr = corr;
          ++kv;
        }
        if (rec.flags & 2) {   // last item: finish the work item
          if (prev >= 0) ok = issue_pv(prev, prev_corr);
          if (!ok) break;
          prev = -1;
          umma_commit(smem_u32(&q_empty[qs]));
          if (need_ofree) {
            ok = mbar_wait(smem_u32(o_free), (wi - 1) & 1, wc);
            need_ofree = false;
          }
          umma_commit(smem_u32(o_full));
          ++wi;
        }
      }
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, wc, false);
    }
  } else {
    // ======================= softmax + epilogue ============================
    // Eight warps: warp w serves TMEM lane quarter w % 4 (query rows
    // 32*(w%4) .. +31) and key half h = (w - 2) / 4 of every S tile (64 keys),
    // with its own running max m_h, sum l_h and accumulator O_h.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;           // 0: keys [0, 64), 1: [64, 128)
    const int r = quarter * 32 + lane;          // row of the 128-row chunk
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_tmem = tmem_base + lane_off + C::kOCol + half * 128;
    const float c2 = a.scale_log2;
    int icount = 0, kv = 0, wi = 0;
    bool ok = true;
    Chunk ck{};
    int gq = 0;
    long long row = 0, position = 0;
    bool row_valid = false;
    float m_used = kFiniteMin, l = 0.f;   // this half's running max and sum
    int pv_wi = 0;
    bool stored = false;                  // this thread issued output tensor stores
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
        ck = make_chunk(p, rec.w);
        const int P = ck.c * 128 + r;
        gq = P / a.tile_q;
        row = (long long)ck.t * a.tile_q + P % a.tile_q;
        position = (long long)a.offset + row;
        row_valid = row < a.valid_lq;
        m_used = kFiniteMin;
        l = 0.f;
        pv_wi = 0;
      }
      if (rec.kind != KIND_EMPTY) {
        const int st = kv % kStages;
        const uint32_t par = (kv / kStages) & 1;
        ok = mbar_wait(smem_u32(&s_full[st]), par, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t s_tmem = tmem_base + lane_off + C::kSCol + st * 128 + half * 64;
        uint32_t s[2][32];
        tmem_ld32(s_tmem, s[0]);
        tmem_ld32(s_tmem + 32, s[1]);
        tmem_wait_ld();
        reg_fence(s[0]);
        reg_fence(s[1]);
        // validity of this warp's 64 entries; a mixed warp masks on every lane
        float bias = 0.f;
        uint32_t vm0 = 0xffffffffu, vm1 = 0xffffffffu;
        bool full = true;
        if (rec.kind == KIND_SEL) {
          const long long ks = rec.kstart + half * 64;
          const bool row_full = row_valid && ks + 63 <= position && ks + 63 < a.valid_lk;
          full = __all_sync(0xffffffffu, row_full);
          if (!full) {
            const long long lim = row_valid ? min(position + 1, (long long)a.valid_lk) - ks : 0;
            vm0 = lim >= 32 ? 0xffffffffu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
            const long long lim1 = lim - 32;
            vm1 = lim1 >= 32 ? 0xffffffffu : (lim1 <= 0 ? 0u : ((1u << lim1) - 1u));
          }
        } else if (rec.kind == KIND_POOL) {
          bias = a.corr_shift;
          full = false;
          vm0 = rec.mask[2 * half];
          vm1 = rec.mask[2 * half + 1];
        } else {   // KIND_CORR (at most 64 entries: half 1 is all masked)
          bias = a.corr_shift;
          const int nv = rec.nvalid - half * 64;
          full = nv >= 64;
          if (!full) {
            vm0 = nv >= 32 ? 0xffffffffu : (nv <= 0 ? 0u : ((1u << nv) - 1u));
            const int nv1 = nv - 32;
            vm1 = nv1 >= 32 ? 0xffffffffu : (nv1 <= 0 ? 0u : ((1u << nv1) - 1u));
          }
        }
        // Full warps keep the raw scores (c2 > 0 keeps the order; x = s*c2 + bias
        // is formed inside the exponent); a warp with any invalid entry forms
        // x = s*c2 + bias and gives masked entries finite_min, exactly as the
        // reference kernel masks its logits.
        float mt;
        if (!full) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x0 = fmaf(__uint_as_float(s[0][j]), c2, bias);
            const float x1 = fmaf(__uint_as_float(s[1][j]), c2, bias);
            s[0][j] = ((vm0 >> j) & 1u) ? __float_as_uint(x0) : __float_as_uint(kFiniteMin);
            s[1][j] = ((vm1 >> j) & 1u) ? __float_as_uint(x1) : __float_as_uint(kFiniteMin);
          }
        }
        {
          float mx0 = max3f(__uint_as_float(s[0][0]), __uint_as_float(s[0][1]), __uint_as_float(s[0][2]));
          float mx1 = max3f(__uint_as_float(s[0][16]), __uint_as_float(s[0][17]), __uint_as_float(s[0][18]));
          float mx2 = max3f(__uint_as_float(s[1][0]), __uint_as_float(s[1][1]), __uint_as_float(s[1][2]));
          float mx3 = max3f(__uint_as_float(s[1][16]), __uint_as_float(s[1][17]), __uint_as_float(s[1][18]));
#pragma unroll
          for (int j = 3; j < 15; j += 2) {
            mx0 = max3f(mx0, __uint_as_float(s[0][j]), __uint_as_float(s[0][j + 1]));
            mx1 = max3f(mx1, __uint_as_float(s[0][16 + j]), __uint_as_float(s[0][17 + j]));
            mx2 = max3f(mx2, __uint_as_float(s[1][j]), __uint_as_float(s[1][j + 1]));
            mx3 = max3f(mx3, __uint_as_float(s[1][16 + j]), __uint_as_float(s[1][17 + j]));
          }
          mx0 = max3f(mx0, __uint_as_float(s[0][15]), mx1);
          mx2 = max3f(mx2, __uint_as_float(s[1][15]), mx3);
          const float m4 = max3f(mx0, mx2, fmaxf(__uint_as_float(s[0][31]), __uint_as_float(s[1][31])));
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
          if (pv_wi > 0) {
            // O_h holds PVs of this work item: wait for the latest one, rescale.
            ok = mbar_wait(smem_u32(pv_done), (kv - 1) & 1, wc);
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
        // P = 2^(x - m): a masked entry (x = finite_min) weighs 1 while the half
        // has seen nothing but masked entries (m = finite_min), else 0.
        // x - m = fma(s, c2, bias - m) for a full warp, fma(x, 1, -m) otherwise (exact);
        // pairs of keys share one packed FMA and one packed add of the row sums.
        const float2 cm2 = full ? make_float2(c2, c2) : make_float2(1.f, 1.f);
        const float2 nb2 = full ? make_float2(bias - m_used, bias - m_used) : make_float2(-m_used, -m_used);
        float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float2 xv = fma_f32x2(
                make_float2(__uint_as_float(s[c][2 * q]), __uint_as_float(s[c][2 * q + 1])), cm2, nb2);
            float2 pv;
            pv.x = ex2(xv.x);
            pv.y = ex2(xv.y);
            rs[q & 3] = add_f32x2(rs[q & 3], pv);
            pk[16 * c + q] = pack_p<VT>(pv.x, pv.y);
          }
        }
        l += ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y));
        // P_h -> the first 32 columns of this half's own S columns (already read)
        tmem_st32(s_tmem, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&p_full[2 * st + half]));
        ++kv;
        ++pv_wi;
      }
      if (rec.flags & 2) {
        // ---- epilogue: combine the halves, out = sum_h a_h O_h / sum_h a_h l_h
        xm[((wi & 1) * 2 + half) * 128 + r] = m_used;
        lsum[((wi & 1) * 2 + half) * 128 + r] = l;
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&lbar[quarter]));
        ok = mbar_wait(smem_u32(&lbar[quarter]), wi & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const float m_o = xm[((wi & 1) * 2 + (half ^ 1)) * 128 + r];
        const float l_o = lsum[((wi & 1) * 2 + (half ^ 1)) * 128 + r];
        const float m_row = fmaxf(m_used, m_o);
        const float a_me = ex2(m_used - m_row), a_o = ex2(m_o - m_row);
        const float lrow = l * a_me + l_o * a_o;
        // (times 2^v_exp[h] when V was scaled into the fp16 range)
        const float vsc = a.v_exp != nullptr ? ldexpf(1.f, a.v_exp[ck.h]) : 1.f;
        const float inv = (pv_wi > 0 && lrow > 0.f) ? vsc / lrow : 0.f;
        const float w_lo = (half == 0 ? a_me : a_o) * inv;   // weight of O_0
        const float w_hi = (half == 0 ? a_o : a_me) * inv;   // weight of O_1
        ok = mbar_wait(smem_u32(o_full), wi & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        // The output tile is staged in this item's Q buffer (its last QK has
        // completed) in the TMA box layout -- rows of 64 columns, 128-byte
        // swizzle -- and written with one coalesced tensor store per 64-column
        // half; the buffer is released to the producer once the store has read it.
        // A segment of a split work item (rec.part >= 0) instead writes its
        // unnormalised output relative to the row maximum m_row, with m_row and
        // the row sum, to its partial slot for attn_combine_kernel.
        const int qs = wi & 1;
        const uint32_t stage = q_smem + qs * C::kTileBytes;
        const uint32_t o0 = tmem_base + lane_off + C::kOCol + half * (D / 2);
        float* part = nullptr;
        if (rec.part >= 0) {
          if (p.split.partials != nullptr && rec.part < p.split.max_slots * kMaxSeg)
            part = p.split.partials + (size_t)rec.part * (128 * D + 256);
          else if (lane == 0)
            atomicOr(p.status, STATUS_BAD_SPLIT);   // bounds check failed: the slot is skipped
        }
#pragma unroll 1
        for (int dc = 0; dc < D / 64; ++dc) {
          uint32_t x0[32], x1[32];
          if (pv_wi > 0) {
            tmem_ld32(o0 + dc * 32, x0);
            tmem_ld32(o0 + 128 + dc * 32, x1);
            tmem_wait_ld();
            reg_fence(x0);
            reg_fence(x1);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) x0[j] = x1[j] = 0u;
          }
          if (part != nullptr) {
            const float a0 = (half == 0 ? a_me : a_o) * vsc, a1 = (half == 0 ? a_o : a_me) * vsc;
            float4* dst = reinterpret_cast<float4*>(part + r * D + half * (D / 2) + dc * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j)
              dst[j] = make_float4(__uint_as_float(x0[4 * j]) * a0 + __uint_as_float(x1[4 * j]) * a1,
                                   __uint_as_float(x0[4 * j + 1]) * a0 + __uint_as_float(x1[4 * j + 1]) * a1,
                                   __uint_as_float(x0[4 * j + 2]) * a0 + __uint_as_float(x1[4 * j + 2]) * a1,
                                   __uint_as_float(x0[4 * j + 3]) * a0 + __uint_as_float(x1[4 * j + 3]) * a1);
            continue;
          }
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float v0 = __uint_as_float(x0[2 * j]) * w_lo + __uint_as_float(x1[2 * j]) * w_hi;
            const float v1 =
                __uint_as_float(x0[2 * j + 1]) * w_lo + __uint_as_float(x1[2 * j + 1]) * w_hi;
            packed[j] = pack2<DT>(v0, v1);
          }
          const int col0 = half * (D / 2) + dc * 32;   // first output column of these 32
          const uint32_t rowb = stage + (col0 / 64) * 16384 + r * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int chunk = ((col0 % 64) >> 3) + j;
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowb + ((chunk ^ (r & 7)) << 4)),
                         "r"(packed[4 * j]), "r"(packed[4 * j + 1]), "r"(packed[4 * j + 2]),
                         "r"(packed[4 * j + 3])
                         : "memory");
          }
        }
        if (part != nullptr && half == 0) {
          part[128 * D + r] = m_row;
          part[128 * D + 128 + r] = lrow;
        }
        fence_proxy_async_smem();
        // D = 128: each half owns one 64-column box (its 4 warps arrive);
        // D = 64: both halves share the box (all 8 warps arrive, half 0 stores).
        const int ob = D == 128 ? half : 0;
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&obar[ob]));
        bool good = true;
        if (part != nullptr) {
          // nothing staged: release the Q buffer with the store path's arrivals
          if (a.out_mc != nullptr) {
            if (lane == 0) mbar_arrive(smem_u32(&q_empty[qs]));
          } else if (quarter == 0 && lane == 0) {
            mbar_arrive(smem_u32(&q_empty[qs]));
          }
        } else if (a.out_mc != nullptr) {
          // Multicast output: every thread of the box's warps copies 16-byte
          // chunks of the staged box (consecutive threads along a row) to the
          // same place of every rank's full output through the NVLink switch.
          good = mbar_wait(smem_u32(&obar[ob]), wi & 1, wc);
          good = __all_sync(0xffffffffu, good);
          if (good) {
            constexpr int kThr = D == 128 ? 128 : 256;
            const int tid = (D == 128 ? 0 : half * 128) + quarter * 32 + lane;
            const int P0 = ck.c * 128;
            for (int kc = tid; kc < 1024; kc += kThr) {
              const int rr = kc >> 3, cc = kc & 7;
              uint4 v;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                           : "r"(stage + ob * 16384 + rr * 128 + ((cc ^ (rr & 7)) << 4)));
              const int P = P0 + rr;
              const long long head = a.mc_head_offset + ck.h * a.G + P / a.tile_q;
              const long long pos = (long long)ck.t * a.tile_q + P % a.tile_q;
              if (ob * 64 + cc * 8 < a.D) {   // head_dim 96 runs on the 128-wide tiles
                char* dst = reinterpret_cast<char*>(a.out_mc) +
                            ((head * a.Lq_pad + pos) * a.D + ob * 64 + cc * 8) * 2;
                multimem_st16(dst, v);
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&q_empty[qs]));
            stored = true;
          }
        } else if (quarter == 0 && lane == 0) {
          if (D == 128 || half == 0) {
            good = mbar_wait(smem_u32(&obar[ob]), wi & 1, wc);
            if (good) {
              const int P0 = ck.c * 128;
              tma_store_3d(&tmap_o, stage + ob * 16384, ob * 64, ck.t * a.tile_q + P0 % a.tile_q,
                           ck.h * a.G + P0 / a.tile_q);
              bulk_commit();
              bulk_wait_read();
              stored = true;
            }
          }
          if (good) mbar_arrive(smem_u32(&q_empty[qs]));
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(o_free));
        ++wi;
      }
    }
    if (stored) {   // output stores complete (and visible to the other GPUs) before the CTA retires
      if (a.out_mc != nullptr) asm volatile("fence.acq_rel.sys;" ::: "memory");
      else bulk_wait_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kTmemCols);
}

// Merge the segments of every split work item: per row,
//   out = sum_s 2^(m_s - m) O_s / sum_s 2^(m_s - m) l_s,  m = max_s m_s,
// the same combination the epilogue applies to the two key halves. Grid
// (slot, group of 8 rows); one thread per 8 output columns (one 16-byte store)
// of a row, with the segments' loads unrolled so that they overlap.
template <int D, int DT>
__global__ void __launch_bounds__(8 * (D / 8)) attn_combine_kernel(Params p) {
  const AttnArgs& a = p.a;
  constexpr int kPart = 128 * D + 256;
  constexpr int kGroups = D / 8;
  const int slot = blockIdx.x;
  const int4 rec = p.split.recs[slot];
  const int nseg = min(rec.y, kMaxSeg);
  if (nseg <= 0) return;
  if (rec.x != slot || rec.x >= p.items) {   // bounds check failed: report, skip the slot
    if (threadIdx.x == 0 && blockIdx.y == 0) atomicOr(p.status, STATUS_BAD_SPLIT);
    return;
  }
  const Chunk ck = make_chunk(p, rec.x);
  const float* base = p.split.partials + (size_t)slot * kMaxSeg * kPart;
  const int r = blockIdx.y * 8 + threadIdx.x / kGroups;
  const int c0 = (threadIdx.x % kGroups) * 8;
  float ms[kMaxSeg], ls[kMaxSeg];
  float m = kFiniteMin;
#pragma unroll
  for (int sg = 0; sg < kMaxSeg; ++sg) {
    ms[sg] = sg < nseg ? base[(size_t)sg * kPart + 128 * D + r] : kFiniteMin;
    ls[sg] = sg < nseg ? base[(size_t)sg * kPart + 128 * D + 128 + r] : 0.f;
    m = fmaxf(m, ms[sg]);
  }
  float den = 0.f, acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
  for (int sg = 0; sg < kMaxSeg; ++sg) {
    if (sg < nseg) {
      const float* ps = base + (size_t)sg * kPart + r * D + c0;
      const float wgt = ex2(ms[sg] - m);
      den = fmaf(wgt, ls[sg], den);
      const float4 u0 = *reinterpret_cast<const float4*>(ps);
      const float4 u1 = *reinterpret_cast<const float4*>(ps + 4);
      acc[0] = fmaf(wgt, u0.x, acc[0]);
      acc[1] = fmaf(wgt, u0.y, acc[1]);
      acc[2] = fmaf(wgt, u0.z, acc[2]);
      acc[3] = fmaf(wgt, u0.w, acc[3]);
      acc[4] = fmaf(wgt, u1.x, acc[4]);
      acc[5] = fmaf(wgt, u1.y, acc[5]);
      acc[6] = fmaf(wgt, u1.z, acc[6]);
      acc[7] = fmaf(wgt, u1.w, acc[7]);
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const uint4 v = make_uint4(pack2<DT>(acc[0] * inv, acc[1] * inv), pack2<DT>(acc[2] * inv, acc[3] * inv),
                             pack2<DT>(acc[4] * inv, acc[5] * inv), pack2<DT>(acc[6] * inv, acc[7] * inv));
  const int P = ck.c * 128 + r;
  const long long head = (long long)ck.h * a.G + P / a.tile_q;
  const long long pos = (long long)ck.t * a.tile_q + P % a.tile_q;
  if (c0 < a.D) {   // head_dim 96 runs on the 128-wide tiles
    if (a.out_mc != nullptr) {
      multimem_st16(reinterpret_cast<char*>(a.out_mc) +
                        (((head + a.mc_head_offset) * a.Lq_pad + pos) * a.D + c0) * 2, v);
      asm volatile("fence.acq_rel.sys;" ::: "memory");
    } else {
      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.out) + ((head * a.Lq_pad + pos) * a.D + c0) * 2) = v;
    }
  }
}

template <int D>
size_t smem_bytes() {
  return 1024 + (size_t)(2 + 2 * kStages) * Cfg<D>::kTileBytes + sizeof(Rec) * kRecs +
         4 * kMaskWordsMax + 4 * (4 * 128 + 4 * 128) + 8 * (4 + 2 * kRecs + 7 * kStages + 10) + 16;
}

}  // namespace

bool attn_tc_supported(const AttnArgs& a) {
  if (a.dt != DT_BF16 && a.dt != DT_F16) return false;
  if (a.D != 64 && a.D != 96 && a.D != 128) return false;
  if (a.pooled_dt != a.dt && a.pooled_dt != DT_F32) return false;
  if (a.block_k % 128 != 0) return false;
  if (!(a.scale_log2 > 0.f)) return false;
  if (a.Nb > 32 * kMaskWordsMax) return false;
  const int R = a.G * a.tile_q;
  if (R % 128 != 0) return false;
  if (a.tile_q % 128 != 0 && 128 % a.tile_q != 0) return false;
  if (a.block_table != nullptr) {   // pages of whole 8-row swizzle atoms, tiles within or across pages
    if (a.page_size < 8 || a.page_size % 8 != 0) return false;
    if (128 % a.page_size != 0 && a.page_size % 128 != 0) return false;
    if (a.num_pages <= 0 || a.table_len <= 0) return false;
    if ((long long)a.table_len * a.page_size < a.Lk_pad) return false;
  }
  return true;
}

// Tensor maps of one attention call: q, k, v, pooled k, pooled v, out.
bool encode_attn_maps(const AttnArgs& a, CUtensorMap (&m)[6]) {
  const int box_rows = a.tile_q >= 128 ? 128 : a.tile_q;
  const int box_heads = 128 / box_rows;
  if (!encode_tmap_3d(&m[0], a.q, a.dt, a.D, a.Lq_pad, a.Hq, 64, box_rows, box_heads))
    return false;
  // (with a multicast output the local tensor map is unused; q stands in for it)
  if (!encode_tmap_3d(&m[5], a.out_mc != nullptr ? a.q : a.out, a.dt, a.D, a.Lq_pad, a.Hq, 64,
                      box_rows, box_heads))
    return false;
  if (a.block_table != nullptr) {   // page pools [pages, page_size, Hkv, D]
    const uint32_t rows = (uint32_t)std::min(a.page_size, 128);
    if (!encode_tmap_pages(&m[1], a.k, a.dt, a.D, a.Hkv, a.page_size, a.num_pages, rows) ||
        !encode_tmap_pages(&m[2], a.v, a.dt, a.D, a.Hkv, a.page_size, a.num_pages, rows))
      return false;
  } else {
    if (!encode_tmap_3d(&m[1], a.k, a.dt, a.D, a.Lk_pad, a.Hkv, 64, 128, 1)) return false;
    if (a.v_conv == nullptr &&
        !encode_tmap_3d(&m[2], a.v, a.dt, a.D, a.Lk_pad, a.Hkv, 64, 128, 1))
      return false;
  }
  const int vdt = a.vdt < 0 ? a.dt : a.vdt;
  if (a.v_conv != nullptr &&   // converted V copy: contiguous [Hkv, Lk_pad, D]
      !encode_tmap_3d(&m[2], a.v_conv, vdt, a.D, a.Lk_pad, a.Hkv, 64, 128, 1))
    return false;
  // Pooled tiles (only read when pooled K/V share the compute dtype).
  const bool pooled_ok = a.corr && a.pooled_dt == a.dt;
  // (pooled tiles unused: q stands in for the pooled tensors)
  if (!encode_tmap_3d(&m[3], pooled_ok ? a.pk : a.q, a.dt, a.D, pooled_ok ? a.Nb : a.Lq_pad,
                      pooled_ok ? a.Hkv : a.Hq, 64, 128, 1))
    return false;
  const void* pvsrc = pooled_ok ? (a.pv_conv != nullptr ? a.pv_conv : a.pv) : a.q;
  if (!encode_tmap_3d(&m[4], pvsrc, pooled_ok && a.pv_conv != nullptr ? vdt : a.dt, a.D,
                      pooled_ok ? a.Nb : a.Lq_pad, pooled_ok ? a.Hkv : a.Hq, 64, 128, 1))
    return false;
  return true;
}

namespace {

// Byte layout of the split scratch inside the caller's workspace.
struct SplitLayout {
  int max_slots = 0;
  size_t recs = 0, parts = 0, clear = 0, total = 0;
};

SplitLayout split_layout(int max_slots, int Dt) {
  auto up = [](size_t x, size_t al) { return (x + al - 1) / al * al; };
  SplitLayout s;
  s.max_slots = max_slots;
  s.recs = 16;       // after the 16-byte work counter
  s.clear = s.recs + 16 * (size_t)max_slots;   // zeroed before each launch
  s.parts = up(s.clear, 256);
  s.total = s.parts + 4 * (size_t)max_slots * kMaxSeg * (128 * Dt + 256);
  return s;
}

int split_tile_width(const AttnArgs& a) { return a.D <= 64 ? 64 : 128; }

}  // namespace

size_t attn_tc_workspace_bytes(const AttnArgs& a) {
  if (!attn_tc_supported(a) || attn_pair_supported(a)) return kAttnMinWorkspace;
  const int nch = (a.G * a.tile_q) / 128;
  const int items = a.Hkv * a.Nt * nch;
  // the latest four tiles of every KV head (the dense tail and its neighbours)
  const int slots = std::min(items, 4 * a.Hkv * nch);
  if (slots <= 0) return kAttnMinWorkspace;
  return std::max(split_layout(slots, split_tile_width(a)).total, (size_t)kAttnMinWorkspace);
}

namespace {

cudaError_t launch_attn_tc_impl(const AttnArgs& a, const TcLaunch& L, void* workspace,
                                int64_t workspace_bytes, cudaStream_t stream) {
  Params p;
  p.a = a;
  p.nch = (a.G * a.tile_q) / 128;
  p.items = a.Hkv * a.Nt * p.nch;
  const int fmt = a.dt == DT_BF16 ? 1 : 0;
  const int vdt = a.vdt < 0 ? a.dt : a.vdt;
  p.idesc_qk = umma_idesc_f16(fmt, 128, 128, 0, 0);
  p.idesc_qk64 = umma_idesc_f16(fmt, 128, 64, 0, 0);
  p.idesc_pv = umma_idesc_f16(vdt == DT_BF16 ? 1 : 0, 128, a.D, 0, 1);
  int* sched = (workspace != nullptr && workspace_bytes >= (int64_t)sizeof(int))
                   ? reinterpret_cast<int*>(workspace)
                   : nullptr;
  p.sched = sched;
  p.status = L.status;
  p.budget = L.budget;
  p.split = Split{};
  if (p.items == 0) return cudaSuccess;

  // KV-segment split when the work items are few per SM (so that one long item
  // outlasts an SM's share of the rest) and the workspace holds the scratch.
  SplitLayout sl;
  const bool few_items = p.items < 32 * L.num_sms;
  if (few_items && sched != nullptr && reinterpret_cast<uintptr_t>(workspace) % 256 == 0) {
    int slots = std::min(p.items, 4 * a.Hkv * p.nch);
    while (slots > 0 && split_layout(slots, split_tile_width(a)).total > (size_t)workspace_bytes)
      slots /= 2;
    if (slots > 0) {
      sl = split_layout(slots, split_tile_width(a));
      char* base = reinterpret_cast<char*>(workspace);
      p.split.recs = reinterpret_cast<int4*>(base + sl.recs);
      p.split.partials = reinterpret_cast<float*>(base + sl.parts);
      p.split.max_slots = sl.max_slots;
    }
  }

  CUtensorMap m[6];
  if (!encode_attn_maps(a, m)) return cudaErrorInvalidValue;
  const int grid = max(1, min(L.num_sms, p.items + p.split.max_slots * (kMaxSeg - 1)));
  cudaError_t e = cudaSuccess;
  if (sched != nullptr) {
    e = cudaMemsetAsync(sched, 0, p.split.max_slots > 0 ? sl.clear : sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  const dim3 cgrid(std::max(1, p.split.max_slots), 16);
  const bool gather = a.corr && a.pooled_dt != a.dt;   // float32 pooled K/V
#define FPV2_ATTN_LAUNCH(DD, TT, VV, GG)                                                    \
  {                                                                                         \
    const size_t smem = smem_bytes<DD>();                                                   \
    e = cudaFuncSetAttribute(attn_tc_kernel<DD, TT, VV, GG>,                                \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);       \
    if (e != cudaSuccess) return e;                                                         \
    attn_tc_kernel<DD, TT, VV, GG><<<grid, kThreads, smem, stream>>>(m[0], m[1], m[2], m[3], m[4], m[5], p); \
    count_launch();                                                                         \
    if (p.split.max_slots > 0) {                                                            \
      attn_combine_kernel<DD, TT><<<cgrid, DD, 0, stream>>>(p);                             \
      count_launch();                                                                       \
    }                                                                                       \
  }
#define FPV2_ATTN_TYPES(DD)                                                                 \
  {                                                                                         \
    if (a.dt == DT_BF16 && vdt == DT_F16) {                                                 \
      if (gather) FPV2_ATTN_LAUNCH(DD, DT_BF16, DT_F16, true)                               \
      else FPV2_ATTN_LAUNCH(DD, DT_BF16, DT_F16, false)                                     \
    } else if (a.dt == DT_BF16 && vdt == DT_BF16) {                                         \
      if (gather) FPV2_ATTN_LAUNCH(DD, DT_BF16, DT_BF16, true)                              \
      else FPV2_ATTN_LAUNCH(DD, DT_BF16, DT_BF16, false)                                    \
    } else if (a.dt == DT_F16 && vdt == DT_F16) {                                           \
      if (gather) FPV2_ATTN_LAUNCH(DD, DT_F16, DT_F16, true)                                \
      else FPV2_ATTN_LAUNCH(DD, DT_F16, DT_F16, false)                                      \
    } else {                                                                                \
      return cudaErrorInvalidValue;                                                         \
    }                                                                                       \
  }
  if (a.D == 64) FPV2_ATTN_TYPES(64)
  // head_dim 96 runs on the 128-wide tiles: the tensor maps have the real
  // extent, so TMA fills columns 96..127 of Q/K/V with zeros (QK unchanged),
  // PV runs with N = 96, and the output store clips at column 96.
  else if (a.D >= 96) FPV2_ATTN_TYPES(128)
  else return cudaErrorInvalidValue;
#undef FPV2_ATTN_TYPES
#undef FPV2_ATTN_LAUNCH
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attn_tc(const AttnArgs& a, const TcLaunch& L, void* workspace,
                           int64_t workspace_bytes, cudaStream_t stream) {
  if (attn_pair_supported(a)) {
    int* sched = (workspace != nullptr && workspace_bytes >= (int64_t)sizeof(int))
                     ? reinterpret_cast<int*>(workspace)
                     : nullptr;
    return launch_attn_pair(a, L, sched, stream);
  }
  return launch_attn_tc_impl(a, L, workspace, workspace_bytes, stream);
}

}  // namespace fpv2
