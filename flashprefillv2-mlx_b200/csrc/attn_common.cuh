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
  int flags;      // bit 0: first item of the work item, bit 1: last item
  int w;          // work item index
  uint32_t mask[4];   // POOL: entry e is a pruned block when bit (e & 31) of mask[e >> 5]
};


struct Params {
  AttnArgs a;
  int nch;          // 128-row chunks per tile
  int items;        // total work items
  uint32_t idesc_qk, idesc_pv;
  int* sched;       // work counter (zeroed before launch); null = static round robin
  int* status;
  long long budget;
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

}  // namespace
}  // namespace fpv2
