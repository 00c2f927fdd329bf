// Launcher interfaces between the C-ABI layer (capi.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fpv2 {

// ---- pooling (pool.cu) ----------------------------------------------------
struct PoolArgs {
  const void* x[2];
  void* out[2];
  int64_t heads, length;
  int D, bs;
};
cudaError_t launch_pool(const PoolArgs& a, int ntensors, int dt_in, int dt_out,
                        cudaStream_t stream);

// Block means of a sequence whose rows live in a page pool [pages, page_size,
// heads, D]: out [heads, length / bs, D], the same exact definition as above.
struct PagedPoolArgs {
  const void* pages;
  const int32_t* table;
  int table_len, num_pages, page_size, heads, D, length, bs;
  void* out;
};
cudaError_t launch_pool_pages(const PagedPoolArgs& a, int dt_in, int dt_out, cudaStream_t stream);

// ---- selection geometry shared by all selection kernels -----------------
// Host-side count of the kernels this library has launched (every launch
// site calls it once per launch; read with fpv2_launch_count).
void count_launch();

struct SelectGeom {
  int Hq, Hkv, G, Lq_pad, Nb, D, Nt;
  int offset, valid_lq, valid_lk;
  int block_k, tile_q, sink, window, last_n;
  float scale, alpha;
};

// Padded lists written by the selection kernels (all null = not written).
struct SelectLists {
  int32_t* sel_ids;
  int32_t* sel_counts;
  int32_t* pr_ids;
  int32_t* pr_counts;
};

// ---- generic (CUDA-core) kernels (generic.cu) ------------------------------
// Mask (nullable) and lists (nullable) for every (kv head, tile); any dtype of
// q / pooled_k, any head_dim.
cudaError_t launch_select_generic(const SelectGeom& g, const void* q, int q_dt, const void* pk,
                                  int pk_dt, uint8_t* mask, const SelectLists& lists,
                                  cudaStream_t stream);
// Unmasked scale * q . pooled_k for every row and block.
cudaError_t launch_raw_scores(const SelectGeom& g, const void* q, int q_dt, const void* pk,
                              int pk_dt, float* out, cudaStream_t stream);
// Mask -> lists.
cudaError_t launch_compact(const uint8_t* mask, int Hkv, int Nt, int Nb, int block_k, int tile_q,
                           int offset, int valid_lk, int32_t* sel_ids, int32_t* sel_counts,
                           int32_t* pr_ids, int32_t* pr_counts, cudaStream_t stream);

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* pk;
  const void* pv;
  int pooled_dt;
  const int32_t* sel_ids;
  const int32_t* sel_counts;
  const int32_t* pr_ids;
  const int32_t* pr_counts;
  void* out;
  int dt;
  int Hq, Hkv, G, Lq_pad, Lk_pad, D, Nt, Nb;
  int offset, valid_lq, valid_lk, block_k, tile_q, corr;
  float scale_log2;   // scale * log2(e)
  float corr_shift;   // log2(block_k)
  // Optional multicast output: the NVLink multicast address of a full
  // [mc_heads, Lq_pad, D] output shared by every rank; this call's query head
  // hq lands at head mc_head_offset + hq. Null: write `out` only.
  void* out_mc = nullptr;
  int mc_head_offset = 0;
  int mc_heads = 0;
  // Optional paged K/V: k and v point at page pools [num_pages, page_size, Hkv,
  // D]; key position p is row p % page_size of page block_table[p / page_size].
  // Null: k and v are [Hkv, Lk_pad, D].
  const int32_t* block_table = nullptr;
  int page_size = 0;
  int num_pages = 0;
  int table_len = 0;
  // Operand type of the P.V product (-1: the input dtype). For bf16 inputs the
  // tcgen05 kernels can run P.V in fp16 -- P rounded to 11 significant bits
  // instead of 8 -- on an exact fp16 copy of V: v_conv [Hkv, Lk_pad, D] and
  // pooled_v_conv [Hkv, Nb, D] (contiguous even when k/v are paged), holding
  // the values times 2^-v_exp[h] (v_exp: per KV head, null = 0); the output is
  // scaled back by 2^v_exp[h].
  int vdt = -1;
  const void* v_conv = nullptr;
  const void* pv_conv = nullptr;
  const int* v_exp = nullptr;
  int* status = nullptr;   // device status word (list bounds reports of debug builds)
};

// ---- V -> fp16 copy for the P.V product (convert.cu) -------------------------
struct VConvArgs {
  const void* v;                 // bf16 [Hkv, L, D], or a page pool [pages, page_size, Hkv, D]
  const int32_t* table;          // page table (null: contiguous v)
  int table_len, num_pages, page_size;
  int Hkv, L, D;
  const void* pv;                // pooled V bf16 [Hkv, Nb, D] (null: none)
  int Nb;
  void* v16;                     // out: fp16 [Hkv, L, D]
  void* pv16;                    // out: fp16 [Hkv, Nb, D]
  int* v_exp;                    // out: [Hkv] power-of-two exponent of the scaling
  unsigned* absmax;              // scratch: [Hkv] (zeroed by the launcher)
};
cudaError_t launch_v_to_f16(const VConvArgs& a, cudaStream_t stream);
// Bytes of the fp16 copies and their scratch (256-byte aligned pieces).
size_t v_conv_bytes(int Hkv, int L, int D, int Nb);
cudaError_t launch_attn_generic(const AttnArgs& a, cudaStream_t stream);

// ---- tcgen05 kernels -------------------------------------------------------
struct TcLaunch {
  int* status;
  long long budget;
  int num_sms;
};

// select_tc.cu: fused score + energy + threshold + lists on tensor cores.
struct SelectTcArgs {
  SelectGeom g;
  int NC;               // query rows per MMA N-chunk (R if R < 128, else 128)
  int box_rows;         // TMA box rows (positions) of one Q chunk
  int box_heads;        // TMA box heads of one Q chunk
  int dt;               // DT_F16 / DT_BF16 (q and pooled_k)
  uint8_t* mask;        // nullable
  int32_t* sel_ids;     // nullable (lists not written)
  int32_t* sel_counts;
  int32_t* pr_ids;
  int32_t* pr_counts;
  int nparts = 1;       // 16-bit parts of the pooled keys ([nparts][Hkv][Nb][D]; 3: float32 keys)
  const int* k_exp = nullptr;   // nparts == 3: per-KV-head exponent of the parts
};
bool select_tc_supported(const SelectGeom& g, int dt);
// float32 pooled keys [Hkv][Nb][D] -> three 16-bit parts [3][Hkv][Nb][D] of dtype
// dt, each head scaled by 2^-k_exp[h] into the type's range (select_tc.cu).
// `out` (256-byte aligned) holds pk_split3_bytes(Hkv, Nb, D); *k_exp points into it.
size_t pk_split3_bytes(int Hkv, int Nb, int D);
cudaError_t launch_pk_split3(const float* pk, void* out, int dt, int Hkv, int Nb, int D,
                             const int** k_exp, cudaStream_t stream);
cudaError_t launch_select_tc(const SelectTcArgs& a, const void* q, const void* pk,
                             const TcLaunch& L, cudaStream_t stream);

// attn_tc.cu: FlashAttention-style block-sparse attention on tensor cores.
// `sched` (nullable) is one int of device scratch used as the work-queue
// counter; it is zeroed on `stream` before the launch. Null = static schedule.
bool attn_tc_supported(const AttnArgs& a);
// `workspace` (nullable, `workspace_bytes` long): its first int is the
// work-queue counter; a workspace of attn_tc_workspace_bytes(a) or more also
// holds the scratch of the KV-segment split of long work items (the partial
// results and their queue), which then runs; a smaller one runs without it.
constexpr size_t kAttnMinWorkspace = 16;
size_t attn_tc_workspace_bytes(const AttnArgs& a);
cudaError_t launch_attn_tc(const AttnArgs& a, const TcLaunch& L, void* workspace,
                           int64_t workspace_bytes, cudaStream_t stream);
// attn_pair.cu: the same with two query chunks of a tile per K/V stream;
// launch_attn_tc routes the shapes it supports (an even number of chunks per
// tile that pair up at the same query positions) to it.
bool attn_pair_supported(const AttnArgs& a);
cudaError_t launch_attn_pair(const AttnArgs& a, const TcLaunch& L, int* sched, cudaStream_t stream);
// Tensor maps of one attention call (attn_tc.cu): q, k, v, pooled k, pooled v, out.
bool encode_attn_maps(const AttnArgs& a, CUtensorMap (&m)[6]);
// attn_wide.cu: the same for head_dim 256 (one softmax warp per row quarter).
bool attn_wide_supported(const AttnArgs& a);
cudaError_t launch_attn_wide(const AttnArgs& a, const TcLaunch& L, int* sched, cudaStream_t stream);

// selftest.cu: bounded-wait failure detection.
cudaError_t launch_wait_selftest(const TcLaunch& L, cudaStream_t stream);

// tensor map helper (capi.cu)
bool encode_tmap_3d(CUtensorMap* map, const void* base, int dt, uint64_t d0, uint64_t d1,
                    uint64_t d2, uint32_t b0, uint32_t b1, uint32_t b2);
// Page pool [pages, page_size, heads, D] as a 4-D map with dims (D, heads,
// page_size, pages) and a box of 64 features x 1 head x `rows` rows x 1 page.
bool encode_tmap_pages(CUtensorMap* map, const void* base, int dt, uint64_t D, uint64_t heads,
                       uint64_t page_size, uint64_t pages, uint32_t rows);

}  // namespace fpv2
