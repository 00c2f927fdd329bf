// Work items, item records and chunk geometry shared by the block-sparse
// attention kernels (attn_tc.cu: head_dim up to 128; attn_wide.cu: 256).
//
// A work item is one 128-row chunk of a selection tile (the G query heads of
// one KV head packed together); the producer walks its lists
// (fpv2/kernel.py:249-255) and publishes one record per KV item: a 128-key
// sub-tile of a selected block (SEL), a 128-row tile of pooled K/V with a mask
// of the pruned entries in it (POOL), a gathered chunk of float32 pooled rows
// (CORR), or an EMPTY record for a chunk without keys.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace fpv2 {
namespace {

// Lazy-rescale threshold in log2 units: P = 2^(x - m) stays below 2^T, which
// the 16-bit P of the PV product represents (fp16 max 65504 < 2^16).
template <int DT> struct RescaleT { static constexpr float value = 16.0f; };
template <> struct RescaleT<DT_F16> { static constexpr float value = 15.0f; };
constexpr int kMaskWordsMax = 64;           // pooled-entry mask of one work item (Nb <= 2048)

enum : int { KIND_SEL = 0, KIND_POOL = 1, KIND_CORR = 2, KIND_EMPTY = 3, KIND_DONE = 4 };

struct Rec {
  int kind;
  int kstart;     // SEL: first key; POOL: first pooled row; CORR: first list entry
  int nvalid;     // CORR: valid list entries in this chunk
  int flags;      // bit 0: first item of the work unit, bit 1: last item
  int w;          // work item index
  int part;       // -1: the unit is a whole work item; else its partial-result slot
  uint32_t mask[4];   // POOL: entry e is a pruned block when bit (e & 31) of mask[e >> 5]
};

// KV-segment split of long work items (attn_tc_kernel). The work counter first
// walks kMaxSeg units (w, s) for each of the first max_slots work items (the
// latest tiles, whose causal extent is largest) and then the remaining items
// one unit each. An item with more than 2 * kSegLen KV items is cut into
// nseg = min(kMaxSeg, ceil(n / kSegLen)) contiguous segments of its KV item
// sequence; unit (w, s < nseg) runs segment s and writes its unnormalised
// output with its row maxima and sums to slot w * kMaxSeg + s, and
// attn_combine_kernel merges the segments. Units that an item does not need
// (s >= nseg, or s > 0 for a short item, which unit (w, 0) runs whole) are
// skipped after the item's list walk. Which items split depends only on the
// lists, never on timing.
constexpr int kMaxSeg = 16;
constexpr int kSegLen = 64;     // target KV items per segment

struct Split {
  int4* recs;          // [max_slots] (w, nseg, 0, 0); nseg 0 = not split (zeroed before launch)
  float* partials;     // [max_slots][kMaxSeg][128 * Dt + 256]: O rows, then m[128], l[128]
  int max_slots;       // 0: no split
};


struct Params {
  AttnArgs a;
  int nch;          // 128-row chunks per tile
  int items;        // total work items
  uint32_t idesc_qk, idesc_pv;
  uint32_t idesc_qk64;  // Q.K^T with N = 64 (the two key parts of a gathered CORR item)
  int* sched;       // work counter (zeroed before launch); null = static round robin
  int* status;
  long long budget;
  Split split;      // attn_tc_kernel only
};

struct Chunk {
  int h, t, c;
  int g0, p0;               // first head / position of the chunk inside the tile
  long long abs_last;       // last valid absolute query position of the chunk
};

__device__ __forceinline__ Chunk make_chunk(const Params& p, int w) {
  const AttnArgs& a = p.a;
  Chunk ck;
  const int per_t = a.Hkv * p.nch;
  ck.t = a.Nt - 1 - w / per_t;   // latest tiles (most causal work) first
  const int r = w % per_t;
  ck.h = r / p.nch;
  ck.c = r % p.nch;
  const int P0 = ck.c * 128;
  ck.g0 = P0 / a.tile_q;
  ck.p0 = P0 % a.tile_q;
  const long long span = min(a.tile_q, 128);
  const long long last_row =
      min((long long)ck.t * a.tile_q + ck.p0 + span, (long long)a.valid_lq) - 1;
  ck.abs_last = (long long)a.offset + last_row;
  return ck;
}

__device__ __forceinline__ int clampi(int x, int lo, int hi) { return min(max(x, lo), hi); }

// Register budget of a warpgroup (setmaxnreg; all four warps execute it).
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Bits 0 .. n-1 set (n clamped to [0, 32]).
__device__ __forceinline__ uint32_t prefix_mask(long long n) {
  return n >= 32 ? 0xffffffffu : (n <= 0 ? 0u : ((1u << n) - 1u));
}

}  // namespace
}  // namespace fpv2
