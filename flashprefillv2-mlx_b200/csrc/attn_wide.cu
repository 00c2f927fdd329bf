// Block-sparse attention on tensor cores for head_dim 256 (tcgen05 + TMEM + TMA).
//
// Same math and work items as attn_tc.cu (fpv2/kernel.py:187-414): per KV item
//   S[128x128] = Q . K^T      tcgen05.mma SS over a contraction of 256 (16 K16
//                             steps), fp32 in TMEM, double buffered
//   P = 2^(S*c - m)           one softmax warp per TMEM lane quarter: a thread
//                             owns one query row and all 128 keys, so each row
//                             has a single running max m and sum l
//   O[128x256] += P . V       tcgen05.mma TS with N = 256 (A = P from TMEM)
// TMEM = O (256 columns) | S buffer 0 | S buffer 1. A 256-wide Q, K or V tile
// is 64 KB, so Q, K and V are single-buffered in shared memory: the next K tile
// loads once the QK reading the current one completes, the next V tile once the
// PV completes, and the next work item's Q once its last QK completes. The
// output tile is staged in the V buffer (free after the work item's last PV)
// and written with TMA stores, or with NVLink multicast stores.
//
// Warp roles (192 threads, one persistent CTA per SM):
//   warp 0     producer (work items from a global counter, lists, TMA loads);
//   warp 1     MMA issuer;
//   warps 2-5  softmax and the output epilogue, warp w on TMEM lane quarter w % 4.
#include "attn_common.cuh"

namespace fpv2 {

namespace {

constexpr int kD = 256;
constexpr int kWThreads = 192;
constexpr int kWRecs = 8;
constexpr int kWTmemCols = 512;
constexpr int kBoxes = kD / 64;               // 64-column TMA boxes of a tile
constexpr int kTile = 128 * kD * 2;           // 64 KB
constexpr uint32_t kOCol = 0, kSCol = 256;    // O | S_0 | S_1

// DT: input dtype; VT: operand type of the P.V product (V and P).
template <int DT, int VT>
__global__ void __launch_bounds__(kWThreads, 1)
    attn_wide_kernel(const __grid_constant__ CUtensorMap tmap_q,
                     const __grid_constant__ CUtensorMap tmap_k,
                     const __grid_constant__ CUtensorMap tmap_v,
                     const __grid_constant__ CUtensorMap tmap_pk,
                     const __grid_constant__ CUtensorMap tmap_pv,
                     const __grid_constant__ CUtensorMap tmap_o, Params p) {
  const AttnArgs& a = p.a;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_base);

  const uint32_t q_smem = base;
  const uint32_t k_smem = base + kTile;
  const uint32_t v_smem = base + 2 * kTile;     // also the output staging
  Rec* recs = reinterpret_cast<Rec*>(gbase + 3 * kTile);          // [kWRecs]
  uint32_t* pmask = reinterpret_cast<uint32_t*>(recs + kWRecs);  // producer-private [64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(pmask + kMaskWordsMax);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 1;
  uint64_t* rec_full = q_empty + 1;        // [kWRecs]
  uint64_t* rec_empty = rec_full + kWRecs;
  uint64_t* k_full = rec_empty + kWRecs;
  uint64_t* k_empty = k_full + 1;
  uint64_t* v_full = k_empty + 1;
  uint64_t* v_empty = v_full + 1;
  uint64_t* s_full = v_empty + 1;          // [2]
  uint64_t* p_full = s_full + 2;           // [2] (4 softmax warps)
  uint64_t* pv_done = p_full + 2;
  uint64_t* o_full = pv_done + 1;
  uint64_t* o_free = o_full + 1;           // 4 softmax warps
  uint64_t* staged = o_free + 1;           // output tile staged (4 warps)
  uint64_t* stage_free = staged + 1;       // output stores have read the staging
  uint64_t* drain = stage_free + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool mc = a.out_mc != nullptr;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_empty), 1);        // the work item's last QK
    for (int i = 0; i < kWRecs; ++i) {
      mbar_init(smem_u32(&rec_full[i]), 1);
      mbar_init(smem_u32(&rec_empty[i]), 1 + 4);   // MMA thread + 4 softmax warps
    }
    mbar_init(smem_u32(k_full), 1);
    mbar_init(smem_u32(k_empty), 1);
    mbar_init(smem_u32(v_full), 1);
    mbar_init(smem_u32(v_empty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s_full[i]), 1);
      mbar_init(smem_u32(&p_full[i]), 4);
    }
    mbar_init(smem_u32(pv_done), 1);
    mbar_init(smem_u32(o_full), 1);
    mbar_init(smem_u32(o_free), 4);
    mbar_init(smem_u32(staged), 4);
    mbar_init(smem_u32(stage_free), mc ? 4 : 1);
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kWTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
    tma_prefetch_desc(&tmap_pk);
    tma_prefetch_desc(&tmap_pv);
    tma_prefetch_desc(&tmap_o);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  WaitCtx wc{p.status, abort_flag, p.budget};
  const int bk_sub = a.block_k / 128;
  const bool pool_tiles = a.corr && a.pooled_dt == DT;   // TMA pooled tiles vs gather

  if (warp == 0) {
    // ============================ producer ================================
    int qcount = 0, icount = 0, kv = 0, wstatic = blockIdx.x;
    int staged_items = 0;      // work items with keys whose V loads have started
    bool ok = true;
    bool first_v = false;      // the work item's first V tile is still to come
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
    // The first V tile of a work item waits until the output stores of the
    // previous work item with keys have read the staging (= the V buffer). Only
    // work items with keys stage their output (an EMPTY one writes its zeros
    // directly), so every stage_free phase is waited once, in order.
    auto wait_stage = [&]() -> bool {
      if (!first_v) return true;
      first_v = false;
      bool good = true;
      if (staged_items > 0 && lane == 0)
        good = mbar_wait(smem_u32(stage_free), (staged_items - 1) & 1, wc);
      ++staged_items;
      return __shfl_sync(0xffffffffu, good, 0);
    };
    auto emit = [&](const Rec& rec, const Chunk& ck, long long lrow) -> bool {
      const int ri = icount % kWRecs;
      bool good = true;
      if (lane == 0) good = mbar_wait(smem_u32(&rec_empty[ri]), ((icount / kWRecs) & 1) ^ 1, wc);
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) return false;
      if (lane == 0) {
        recs[ri] = rec;
        mbar_arrive(smem_u32(&rec_full[ri]));
      }
      ++icount;
      if (rec.kind == KIND_EMPTY || rec.kind == KIND_DONE) return true;
      const uint32_t par = (kv & 1) ^ 1;
      if (rec.kind != KIND_CORR) {
        const CUtensorMap* mk = rec.kind == KIND_SEL ? &tmap_k : &tmap_pk;
        const CUtensorMap* mv = rec.kind == KIND_SEL ? &tmap_v : &tmap_pv;
        if (lane == 0) {
          good = mbar_wait(smem_u32(k_empty), par, wc);
          if (good) {
            mbar_arrive_expect_tx(smem_u32(k_full), (uint32_t)kTile);
#pragma unroll
            for (int hh = 0; hh < kBoxes; ++hh)
              tma_load_3d(k_smem + hh * 16384, mk, smem_u32(k_full), hh * 64, rec.kstart, ck.h);
            good = mbar_wait(smem_u32(v_empty), par, wc);
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (good) good = wait_stage();
        if (good && lane == 0) {
          mbar_arrive_expect_tx(smem_u32(v_full), (uint32_t)kTile);
#pragma unroll
          for (int hh = 0; hh < kBoxes; ++hh)
            tma_load_3d(v_smem + hh * 16384, mv, smem_u32(v_full), hh * 64, rec.kstart, ck.h);
        }
        if (!good) return false;
      } else {
        // Float32 pooled inputs: gather up to 64 listed entries in two parts --
        // rows e < 64 hold round(x), rows 64 + e hold round(x - round(x)) -- so
        // that Q.K^T accumulated over both parts carries the float32 pooled keys
        // and P.V over both parts the float32 pooled values; K first (its slot
        // frees with the previous QK), then V (its slot frees with the previous
        // PV, which is issued after this item's QK).
        // (values in the P.V operand type, scaled by 2^-v_exp[h] like the V copy)
        const float vs = a.v_exp != nullptr ? ldexpf(1.f, -a.v_exp[ck.h]) : 1.f;
        auto gather = [&](const void* src_base, uint32_t dst, bool is_v) {
          constexpr int kChunks = kD / 8;   // 16-byte chunks per row
          for (int idx = lane; idx < 128 * kChunks; idx += 32) {
            const int e = idx / kChunks, cidx = idx % kChunks;
            const int hh = cidx >> 3, cc = cidx & 7;
            const uint32_t off = hh * 16384 + e * 128 + ((cc ^ (e & 7)) << 4);
            const int ent = e & 63;
            const bool low = e >= 64;
            uint4 val = make_uint4(0, 0, 0, 0);
            if (ent < rec.nvalid) {
              const int blk = clamp_entry(a.pr_ids[lrow + rec.kstart + ent], 0, a.Nb - 1, p.status);
              const long long src = ((long long)ck.h * a.Nb + blk) * kD + cidx * 8;
              const float4* f = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src_base) + src);
              const float4 x0 = __ldg(f), x1 = __ldg(f + 1);
              if (is_v)
                val = make_uint4(pack2_split<VT>(x0.x * vs, x0.y * vs, low),
                                 pack2_split<VT>(x0.z * vs, x0.w * vs, low),
                                 pack2_split<VT>(x1.x * vs, x1.y * vs, low),
                                 pack2_split<VT>(x1.z * vs, x1.w * vs, low));
              else
                val = make_uint4(pack2_split<DT>(x0.x, x0.y, low), pack2_split<DT>(x0.z, x0.w, low),
                                 pack2_split<DT>(x1.x, x1.y, low), pack2_split<DT>(x1.z, x1.w, low));
            }
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst + off), "r"(val.x),
                         "r"(val.y), "r"(val.z), "r"(val.w)
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
        };
        if (lane == 0) good = mbar_wait(smem_u32(k_empty), par, wc);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) return false;
        gather(a.pk, k_smem, false);
        if (lane == 0) mbar_arrive(smem_u32(k_full));
        if (lane == 0) good = mbar_wait(smem_u32(v_empty), par, wc);
        good = __shfl_sync(0xffffffffu, good, 0);
        if (good) good = wait_stage();
        if (!good) return false;
        gather(a.pv, v_smem, true);
        if (lane == 0) mbar_arrive(smem_u32(v_full));
      }
      ++kv;
      return true;
    };

    for (int w = next_work(); w < p.items && ok; w = next_work()) {
      const Chunk ck = make_chunk(p, w);
      const long long lrow = ((long long)ck.h * a.Nt + ck.t) * a.Nb;
      const int nsel = clamp_entry(a.sel_counts[(long long)ck.h * a.Nt + ck.t], 0, a.Nb, p.status);
      const int npr = a.corr ? clamp_entry(a.pr_counts[(long long)ck.h * a.Nt + ck.t], 0, a.Nb, p.status) : 0;
      first_v = true;
      // Q tile of the chunk (its buffer frees when the previous item's last QK completes).
      if (lane == 0) ok = mbar_wait(smem_u32(q_empty), (qcount & 1) ^ 1, wc);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(smem_u32(q_full), (uint32_t)kTile);
#pragma unroll
        for (int hh = 0; hh < kBoxes; ++hh)
          tma_load_3d(q_smem + hh * 16384, &tmap_q, smem_u32(q_full), hh * 64,
                      ck.t * a.tile_q + ck.p0, ck.h * a.G + ck.g0);
      }
      ++qcount;
      // Selected blocks up to the first one past the chunk (fpv2/kernel.py:249-255).
      int n_sel_items = 0, brk = nsel;
      for (int i0 = 0; i0 < nsel; i0 += 32) {
        const int i = i0 + lane;
        const bool in = i < nsel;
        const int blk = in ? clamp_entry(a.sel_ids[lrow + i], 0, a.Nb - 1, p.status) : 0;
        const long long bstart = (long long)blk * a.block_k;
        const unsigned stop = __ballot_sync(0xffffffffu, in && bstart > ck.abs_last);
        const int lim = stop ? (__ffs(stop) - 1) : 32;
        int contrib = 0;
        if (in && lane < lim) contrib = (int)min((long long)bk_sub, (ck.abs_last - bstart) / 128 + 1);
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
          for (int y = 0; y < 4 && w0 + y < nwords; ++y) any |= pmask[w0 + y];
          n_corr_items += any != 0u;
        }
      } else if (npr > 0) {
        n_corr_items = (npr + 63) / 64;   // 64 entries (high + low parts) per item
      }
      const int n_items = max(1, n_sel_items + n_corr_items);
      int emitted = 0;
      auto make_rec = [&](int kind, int kstart, int nvalid) {
        Rec r;
        r.kind = kind;
        r.kstart = kstart;
        r.nvalid = nvalid;
        r.flags = (emitted == 0 ? 1 : 0) | (emitted == n_items - 1 ? 2 : 0);
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
            if (ks > ck.abs_last) break;
            ok = emit(make_rec(KIND_SEL, (int)ks, 0), ck, lrow);
          }
        }
      }
      if (pool_tiles) {
        const int nwords = (a.Nb + 31) / 32;
        for (int j = 0; j < n_ptiles && ok && npr > 0; ++j) {
          uint32_t m4[4];
          uint32_t any = 0;
#pragma unroll
          for (int y = 0; y < 4; ++y) {
            m4[y] = (4 * j + y < nwords) ? pmask[4 * j + y] : 0u;
            any |= m4[y];
          }
          if (!any) continue;
          Rec r = make_rec(KIND_POOL, j * 128, 0);
#pragma unroll
          for (int y = 0; y < 4; ++y) r.mask[y] = m4[y];
          ok = emit(r, ck, lrow);
        }
        __syncwarp();   // mask reads done before the next work item clears it
      } else {
        for (int j = 0; j < n_corr_items && ok; ++j)
          ok = emit(make_rec(KIND_CORR, j * 64, min(64, npr - j * 64)), ck, lrow);
      }
      if (ok && n_sel_items + n_corr_items == 0) ok = emit(make_rec(KIND_EMPTY, 0, 0), ck, lrow);
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
      if (kv > 0) {
        mbar_wait(smem_u32(k_full), (kv - 1) & 1, wc, false);
        mbar_wait(smem_u32(v_full), (kv - 1) & 1, wc, false);
      }
      if (qcount > 0) mbar_wait(smem_u32(q_full), (qcount - 1) & 1, wc, false);
    }
  } else if (warp == 1) {
    // ============================ MMA issuer ==============================
    // Per record: QK(k) into S buffer k % 2, then PV(k-1) -- the products of two
    // consecutive KV items overlap the softmax of the one in between.
    if (lane == 0) {
      int qcount = 0, icount = 0, kv = 0, wi = 0;
      bool ok = true, need_ofree = false, first_pv = true, need_q = false;
      int prev = -1;   // kv index whose PV is pending
      bool prev_last = false;   // that PV closes its work item
      bool prev_corr = false;   // that item is a gathered CORR item (high + low parts)
      auto issue_pv = [&](int n, bool last, bool corr) -> bool {
        const int st = n & 1;
        if (!mbar_wait(smem_u32(v_full), n & 1, wc)) return false;
        if (!mbar_wait(smem_u32(&p_full[st]), (n >> 1) & 1, wc)) return false;
        if (need_ofree) {
          if (!mbar_wait(smem_u32(o_free), (wi - 1) & 1, wc)) return false;
          need_ofree = false;
        }
        tc_fence_after();
        // O[128 x 256] += P V: P (128 keys as 16-bit pairs) in the first 64
        // columns of the S buffer, V MN-major in four 64-column boxes. A CORR
        // item's P (64 entries) multiplies the high value rows 0..63 and then the
        // low value rows 64..127.
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t pcol = corr ? (uint32_t)(kk & 3) * 8 : (uint32_t)kk * 8;
          const uint64_t bdesc = sw128_desc(v_smem + kk * 2048, 16384, 1024);
          umma_ts(tmem_base + kOCol, tmem_base + kSCol + st * 128 + pcol, bdesc, p.idesc_pv,
                  (first_pv && kk == 0) ? 0u : 1u);
        }
        first_pv = false;
        umma_commit(smem_u32(v_empty));
        umma_commit(smem_u32(pv_done));
        if (last) {
          umma_commit(smem_u32(o_full));
          ++wi;
        }
        return true;
      };
      while (ok) {
        const int ri = icount % kWRecs;
        ok = mbar_wait(smem_u32(&rec_full[ri]), (icount / kWRecs) & 1, wc);
        if (!ok) break;
        const Rec rec = recs[ri];
        mbar_arrive(smem_u32(&rec_empty[ri]));
        ++icount;
        if (rec.kind == KIND_DONE) break;
        if (rec.flags & 1) need_q = true;
        if (rec.kind != KIND_EMPTY) {
          const int st = kv & 1;
          // S buffer st held P of item kv - 2, read by a PV issued earlier from
          // this thread: tcgen05.mma ops run in issue order, so no wait here.
          ok = mbar_wait(smem_u32(k_full), kv & 1, wc);
          if (ok && need_q) {
            ok = mbar_wait(smem_u32(q_full), qcount & 1, wc);
            ++qcount;
            need_q = false;
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t s_tmem = tmem_base + kSCol + st * 128;
          const bool corr = rec.kind == KIND_CORR;
          if (!corr) {
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk) {
              const int hh = kk / 4, sub = kk % 4;
              const uint64_t adesc = sw128_desc(q_smem + hh * 16384 + sub * 32, 16, 1024);
              const uint64_t bdesc = sw128_desc(k_smem + hh * 16384 + sub * 32, 16, 1024);
              umma_ss(s_tmem, adesc, bdesc, p.idesc_qk, kk > 0 ? 1u : 0u);
            }
          } else {
            // gathered CORR item: S[:, 0:64] = Q.K_high^T + Q.K_low^T (key rows 0..63
            // and 64..127, 8 KB apart in each 64-column box), N = 64, one accumulator
#pragma unroll
            for (int part = 0; part < 2; ++part) {
#pragma unroll
              for (int kk = 0; kk < kD / 16; ++kk) {
                const int hh = kk / 4, sub = kk % 4;
                const uint64_t adesc = sw128_desc(q_smem + hh * 16384 + sub * 32, 16, 1024);
                const uint64_t bdesc = sw128_desc(k_smem + hh * 16384 + part * 8192 + sub * 32, 16, 1024);
                umma_ss(s_tmem, adesc, bdesc, p.idesc_qk64, (part | kk) ? 1u : 0u);
              }
            }
          }
          umma_commit(smem_u32(&s_full[st]));
          umma_commit(smem_u32(k_empty));
          if (rec.flags & 2) umma_commit(smem_u32(q_empty));   // Q no longer read
          if (prev >= 0) ok = issue_pv(prev, prev_last, prev_corr);
          if (!ok) break;
          if (rec.flags & 1) {
            need_ofree = wi > 0;
            first_pv = true;
          }
          prev = kv;
          prev_last = (rec.flags & 2) != 0;
          prev_corr = corr;
          ++kv;
        } else {
          // EMPTY work item: finish the pending PV, release Q, hand over an O of zeros.
          if (prev >= 0) ok = issue_pv(prev, prev_last, prev_corr);
          if (!ok) break;
          prev = -1;
          if (need_q) {
            ok = mbar_wait(smem_u32(q_full), qcount & 1, wc);
            ++qcount;
            need_q = false;
          }
          if (ok && wi > 0) ok = mbar_wait(smem_u32(o_free), (wi - 1) & 1, wc);
          if (!ok) break;
          need_ofree = false;
          umma_commit(smem_u32(q_empty));
          umma_commit(smem_u32(o_full));
          ++wi;
        }
      }
      if (ok && prev >= 0) issue_pv(prev, prev_last, prev_corr);
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, wc, false);
    }
  } else {
    // ======================= softmax + epilogue ============================
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t o_tmem = tmem_base + lane_off + kOCol;
    const float c2 = a.scale_log2;
    int icount = 0, kv = 0, wi = 0;
    bool ok = true;
    Chunk ck{};
    int gq = 0;
    long long row = 0, position = 0;
    bool row_valid = false;
    float m_used = kFiniteMin, l = 0.f;   // running max (log2 domain) and sum of the row
    int pv_wi = 0;
    bool stored = false;
    while (ok) {
      const int ri = icount % kWRecs;
      ok = mbar_wait(smem_u32(&rec_full[ri]), (icount / kWRecs) & 1, wc);
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
        const int st = kv & 1;
        ok = mbar_wait(smem_u32(&s_full[st]), (kv >> 1) & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const uint32_t s_tmem = tmem_base + lane_off + kSCol + st * 128;
        uint32_t s[4][32];
        tmem_ld32(s_tmem, s[0]);
        tmem_ld32(s_tmem + 32, s[1]);
        tmem_ld32(s_tmem + 64, s[2]);
        tmem_ld32(s_tmem + 96, s[3]);
        tmem_wait_ld();
        reg_fence(s[0]);
        reg_fence(s[1]);
        reg_fence(s[2]);
        reg_fence(s[3]);
        // Validity of the 128 keys; a warp with any invalid entry masks on every lane.
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
            for (int c = 0; c < 4; ++c) {
              const long long n = lim - 32 * c;
              vm[c] = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
            }
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
            for (int c = 0; c < 4; ++c) {
              const int n = rec.nvalid - 32 * c;
              vm[c] = n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
            }
          }
        }
        float mt;
        if (!full) {
          // x = s*c2 + bias in the log2 domain; a masked entry takes finite_min,
          // exactly as the reference kernel masks its logits.
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float xv = fmaf(__uint_as_float(s[c][j]), c2, bias);
              s[c][j] = ((vm[c] >> j) & 1u) ? __float_as_uint(xv) : __float_as_uint(kFiniteMin);
            }
        }
        {
          float mx[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            mx[i] = max3f(__uint_as_float(s[i >> 1][(i & 1) * 16]),
                          __uint_as_float(s[i >> 1][(i & 1) * 16 + 1]),
                          __uint_as_float(s[i >> 1][(i & 1) * 16 + 2]));
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 3; j < 15; j += 2) {
              mx[2 * c] = max3f(mx[2 * c], __uint_as_float(s[c][j]), __uint_as_float(s[c][j + 1]));
              mx[2 * c + 1] =
                  max3f(mx[2 * c + 1], __uint_as_float(s[c][16 + j]), __uint_as_float(s[c][17 + j]));
            }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            mx[2 * c] = max3f(mx[2 * c], __uint_as_float(s[c][15]), __uint_as_float(s[c][31]));
          const float m8 = fmaxf(max3f(mx[0], mx[1], mx[2]), max3f(mx[3], max3f(mx[4], mx[5], mx[6]), mx[7]));
          mt = full ? fmaf(m8, c2, bias) : m8;
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
            // O holds PVs of this work item: wait for the latest one, rescale.
            ok = mbar_wait(smem_u32(pv_done), (kv - 1) & 1, wc);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
#pragma unroll 1
            for (int dc = 0; dc < kD / 32; ++dc) {
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
        // x - m = fma(s, c2, bias - m) for a full warp, fma(x, 1, -m) otherwise (exact);
        // a masked entry (x = finite_min) weighs 1 while the row has seen nothing
        // but masked entries (m = finite_min), else 0.
        const float2 cm2 = full ? make_float2(c2, c2) : make_float2(1.f, 1.f);
        const float2 nb2 = full ? make_float2(bias - m_used, bias - m_used) : make_float2(-m_used, -m_used);
        float2 rs[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
        uint32_t pk0[32], pk1[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float2 xv = fma_f32x2(
                make_float2(__uint_as_float(s[c][2 * q]), __uint_as_float(s[c][2 * q + 1])), cm2, nb2);
            float2 pv;
            pv.x = ex2(xv.x);
            pv.y = ex2(xv.y);
            rs[q & 3] = add_f32x2(rs[q & 3], pv);
            if (c < 2) pk0[16 * c + q] = pack_p<VT>(pv.x, pv.y);
            else pk1[16 * (c - 2) + q] = pack_p<VT>(pv.x, pv.y);
          }
        }
        l += ((rs[0].x + rs[0].y) + (rs[1].x + rs[1].y)) + ((rs[2].x + rs[2].y) + (rs[3].x + rs[3].y));
        // P of keys [0, 128) -> S columns [0, 64) (already read)
        tmem_st32(s_tmem, pk0);
        tmem_st32(s_tmem + 32, pk1);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&p_full[st]));
        ++kv;
        ++pv_wi;
      }
      if ((rec.flags & 2) && pv_wi == 0) {
        // ---- EMPTY work item: its rows are zeros, written straight to global
        // memory (the staging buffer may still be read by the previous stores).
        ok = mbar_wait(smem_u32(o_full), wi & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        const int P = ck.c * 128 + r;
        const long long head = (long long)ck.h * a.G + P / a.tile_q;
        const long long pos = (long long)ck.t * a.tile_q + P % a.tile_q;
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        if (mc) {
          char* dst = reinterpret_cast<char*>(a.out_mc) + ((head + a.mc_head_offset) * a.Lq_pad + pos) * kD * 2;
          for (int cc = 0; cc < kD / 8; ++cc) multimem_st16(dst + cc * 16, z);
          stored = true;
        } else {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.out) + (head * a.Lq_pad + pos) * kD * 2);
          for (int cc = 0; cc < kD / 8; ++cc) dst[cc] = z;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(o_free));
        ++wi;
      } else if (rec.flags & 2) {
        // ---- epilogue: out = O / l staged in the V buffer (the work item's
        // last PV has completed) as four 64-column TMA boxes, 128-byte swizzle.
        // (times 2^v_exp[h] when V was scaled into the fp16 range)
        const float vsc = a.v_exp != nullptr ? ldexpf(1.f, a.v_exp[ck.h]) : 1.f;
        const float inv = l > 0.f ? vsc / l : 0.f;
        ok = mbar_wait(smem_u32(o_full), wi & 1, wc);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int dc = 0; dc < kD / 32; ++dc) {
          uint32_t o[32];
          tmem_ld32(o_tmem + dc * 32, o);
          tmem_wait_ld();
          reg_fence(o);
          uint32_t packed[16];
#pragma unroll
          for (int j = 0; j < 16; ++j)
            packed[j] = pack2<DT>(__uint_as_float(o[2 * j]) * inv, __uint_as_float(o[2 * j + 1]) * inv);
          const int col0 = dc * 32;
          const uint32_t rowb = v_smem + (col0 / 64) * 16384 + r * 128;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int chunk = ((col0 % 64) >> 3) + j;
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowb + ((chunk ^ (r & 7)) << 4)),
                         "r"(packed[4 * j]), "r"(packed[4 * j + 1]), "r"(packed[4 * j + 2]),
                         "r"(packed[4 * j + 3])
                         : "memory");
          }
        }
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(smem_u32(o_free));
          mbar_arrive(smem_u32(staged));
        }
        bool good = true;
        const int P0 = ck.c * 128;
        if (mc) {
          good = mbar_wait(smem_u32(staged), wi & 1, wc);
          good = __all_sync(0xffffffffu, good);
          if (good) {
            const int tid = quarter * 32 + lane;
            for (int kc = tid; kc < 1024 * kBoxes; kc += 128) {
              const int ob = kc >> 10, rr = (kc >> 3) & 127, cc = kc & 7;
              uint4 v;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                           : "r"(v_smem + ob * 16384 + rr * 128 + ((cc ^ (rr & 7)) << 4)));
              const int P = P0 + rr;
              const long long head = a.mc_head_offset + ck.h * a.G + P / a.tile_q;
              const long long pos = (long long)ck.t * a.tile_q + P % a.tile_q;
              char* dst = reinterpret_cast<char*>(a.out_mc) +
                          ((head * a.Lq_pad + pos) * kD + ob * 64 + cc * 8) * 2;
              multimem_st16(dst, v);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(stage_free));
            stored = true;
          }
        } else if (quarter == 0 && lane == 0) {
          good = mbar_wait(smem_u32(staged), wi & 1, wc);
          if (good) {
#pragma unroll
            for (int ob = 0; ob < kBoxes; ++ob)
              tma_store_3d(&tmap_o, v_smem + ob * 16384, ob * 64, ck.t * a.tile_q + P0 % a.tile_q,
                           ck.h * a.G + P0 / a.tile_q);
            bulk_commit();
            bulk_wait_read();
            stored = true;
            mbar_arrive(smem_u32(stage_free));
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
        ++wi;
      }
    }
    if (stored) {   // output stores complete (and visible to the other GPUs) before the CTA retires
      if (mc) asm volatile("fence.acq_rel.sys;" ::: "memory");
      else bulk_wait_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, kWTmemCols);
}

size_t wide_smem_bytes() {
  return 1024 + (size_t)3 * kTile + sizeof(Rec) * kWRecs + 4 * kMaskWordsMax + 8 * 32 + 16;
}

}  // namespace

bool attn_wide_supported(const AttnArgs& a) {
  if (a.dt != DT_BF16 && a.dt != DT_F16) return false;
  if (a.D != kD) return false;
  if (a.block_table != nullptr) return false;   // paged K/V: head_dim up to 128
  if (a.pooled_dt != a.dt && a.pooled_dt != DT_F32) return false;
  if (a.block_k % 128 != 0) return false;
  if (!(a.scale_log2 > 0.f)) return false;
  if (a.Nb > 32 * kMaskWordsMax) return false;
  const int R = a.G * a.tile_q;
  if (R % 128 != 0) return false;
  if (a.tile_q % 128 != 0 && 128 % a.tile_q != 0) return false;
  return true;
}

cudaError_t launch_attn_wide(const AttnArgs& a, const TcLaunch& L, int* sched, cudaStream_t stream) {
  Params p;
  p.a = a;
  p.nch = (a.G * a.tile_q) / 128;
  p.items = a.Hkv * a.Nt * p.nch;
  const int fmt = a.dt == DT_BF16 ? 1 : 0;
  const int vdt = a.vdt < 0 ? a.dt : a.vdt;
  p.idesc_qk = umma_idesc_f16(fmt, 128, 128, 0, 0);
  p.idesc_qk64 = umma_idesc_f16(fmt, 128, 64, 0, 0);
  p.idesc_pv = umma_idesc_f16(vdt == DT_BF16 ? 1 : 0, 128, kD, 0, 1);
  p.sched = sched;
  p.status = L.status;
  p.budget = L.budget;
  if (p.items == 0) return cudaSuccess;

  const int box_rows = a.tile_q >= 128 ? 128 : a.tile_q;
  const int box_heads = 128 / box_rows;
  CUtensorMap tq, tk, tv, tpk, tpv, to;
  if (!encode_tmap_3d(&tq, a.q, a.dt, a.D, a.Lq_pad, a.Hq, 64, box_rows, box_heads))
    return cudaErrorInvalidValue;
  if (!encode_tmap_3d(&to, a.out_mc != nullptr ? a.q : a.out, a.dt, a.D, a.Lq_pad, a.Hq, 64,
                      box_rows, box_heads))
    return cudaErrorInvalidValue;
  if (!encode_tmap_3d(&tk, a.k, a.dt, a.D, a.Lk_pad, a.Hkv, 64, 128, 1)) return cudaErrorInvalidValue;
  if (!encode_tmap_3d(&tv, a.v_conv != nullptr ? a.v_conv : a.v, vdt, a.D, a.Lk_pad, a.Hkv, 64, 128, 1))
    return cudaErrorInvalidValue;
  const bool pooled_ok = a.corr && a.pooled_dt == a.dt;
  if (!encode_tmap_3d(&tpk, pooled_ok ? a.pk : a.k, a.dt, a.D, pooled_ok ? a.Nb : a.Lk_pad, a.Hkv,
                      64, 128, 1))
    return cudaErrorInvalidValue;
  const void* pvsrc = pooled_ok ? (a.pv_conv != nullptr ? a.pv_conv : a.pv)
                                : (a.v_conv != nullptr ? a.v_conv : a.v);
  if (!encode_tmap_3d(&tpv, pvsrc, vdt, a.D, pooled_ok ? a.Nb : a.Lk_pad, a.Hkv, 64, 128, 1))
    return cudaErrorInvalidValue;
  const int grid = max(1, min(L.num_sms, p.items));
  cudaError_t e = cudaSuccess;
  if (sched != nullptr) {
    e = cudaMemsetAsync(sched, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  const size_t smem = wide_smem_bytes();
#define FPV2_WIDE_LAUNCH(TT, VV)                                                            \
  {                                                                                         \
    e = cudaFuncSetAttribute(attn_wide_kernel<TT, VV>,                                      \
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);       \
    if (e != cudaSuccess) return e;                                                         \
    attn_wide_kernel<TT, VV><<<grid, kWThreads, smem, stream>>>(tq, tk, tv, tpk, tpv, to, p); \
    count_launch();                                                                         \
  }
  if (a.dt == DT_BF16 && vdt == DT_F16) FPV2_WIDE_LAUNCH(DT_BF16, DT_F16)
  else if (a.dt == DT_BF16) FPV2_WIDE_LAUNCH(DT_BF16, DT_BF16)
  else FPV2_WIDE_LAUNCH(DT_F16, DT_F16)
#undef FPV2_WIDE_LAUNCH
  return cudaGetLastError();
}

}  // namespace fpv2
