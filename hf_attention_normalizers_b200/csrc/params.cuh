// Kernel-side parameter block shared by every attention kernel (dense, varlen
// and paged layouts) plus the address arithmetic for each layout.
#pragma once

#include "common.cuh"

namespace hfan {

constexpr int kSupSlots = 64;  // support-list slots per query row (sparsemax keeps ~5 keys on N(0, 1) scores)
constexpr int kKeyScanBlock = 4096;  // key counters per block of the key-offset prefix kernels

constexpr int kKeyMaxEntries = 1024;  // longest key segment a warp of the list dK/dV kernel sorts
// sl_flag bits: a row's support list overflowed in the forward (the backward
// runs both tile kernels), or a long key segment could not be served by the
// list kernels (the tile dK/dV kernel runs; dQ still comes from the lists).
constexpr int kListRowOverflow = 1;
constexpr int kListKeyOverflow = 2;

inline int64_t sparse_key_blocks(int64_t nk) { return (nk + kKeyScanBlock - 1) / kKeyScanBlock; }

struct AttnParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  const void* dout;
  void* dq;
  void* dk;
  void* dv;
  float* stats;  // [2][hq][rows_total]
  float* corr;   // [hq][rows_total]

  int64_t q_sb, q_sh, q_st;
  int64_t k_sb, k_sh, k_st;
  int64_t v_sb, v_sh, v_st;
  int64_t o_sb, o_sh, o_st;
  int64_t do_sb, do_sh, do_st;
  int64_t dq_sb, dq_sh, dq_st;
  int64_t dk_sb, dk_sh, dk_st;
  int64_t dv_sb, dv_sh, dv_st;

  int batch, hq, hkv, d;
  int len_q, len_k;      // dense lengths; varlen/paged maxima
  int rows_total;        // stats rows per head
  int64_t rows_k;        // varlen: packed key rows
  const int* cu_q;       // varlen
  const int* cu_k;
  const int* block_table;  // paged
  const int* seq_lens;
  int page_size, max_blocks;
  int64_t num_cache_tokens;
  int paged;
  int lens_only;           // dense K/V whose per-sequence key lengths come from seq_lens
  int tile_lpt;            // tensor-core kernels: hand tiles out longest-first across the whole grid
  int causal_top_left;     // causal mask aligned at the first key (row i sees j <= i) instead of the last
  // Sparse normalizers: key tiles with support, one bit per (query head,
  // sequence, 64-row block, 128-key tile), written by the tensor-core forward
  // and read by the backward to skip tiles whose probabilities are all zero.
  // Word ((h * batch + b) * mask_qb + block) * mask_words + tile / 32; null: none.
  uint32_t* tile_mask;
  int mask_words, mask_qb;
  // Dropout (dense layout, tensor-core kernels): an element survives when the
  // top 24 bits of its generator word are >= drop_thr24 (= ceil(p 2^24); 0: no
  // dropout) and is then scaled by drop_scale = 1 / (1 - p).  The seed is read
  // from device memory (see dropout_keep4 in common.cuh).
  uint32_t drop_thr24;
  float drop_scale;
  const int64_t* drop_seed;
  // Sparse normalizers: w-weighted mean of V per row (input dtype), written by
  // the tensor-core forward and read by its backward (null: not used).
  void* wm;
  int64_t wm_sb, wm_sh, wm_st;
  // Sparse normalizers, tensor-core path without dropout: per-row support
  // lists written by the forward (null: none).  Row r of query head h owns
  // kSupSlots consecutive slots at [(h * rows_total + r) * kSupSlots]: NWG =
  // head_dim / 32 sub-lists (one per row warpgroup, keys in increasing order)
  // of kSupSlots / NWG slots.  sl_ent: {key token (the K/V token index),
  // float bits of p > 0}; sl_g: the backward's dP, then dS; sl_cnt:
  // [(h * rows_total + r) * NWG + w] entries of sub-list w; sl_flag: nonzero
  // when some sub-list overflowed (the backward then runs the tile kernels).
  int2* sl_ent;
  float* sl_g;
  int* sl_cnt;
  int* sl_flag;
  // The same entries transposed to the key side for dK/dV: key id kid =
  // (b * hkv + kvh) * len_k + token (dense) or kvh * rows_k + token (varlen),
  // sl_nk ids.  sl_kcnt: entries per key (then the fill cursor); sl_koff:
  // [sl_nk + 1] exclusive prefix; sl_bsum: per-block sums of the prefix
  // kernels; sl_tr: slot numbers grouped by key, sorted within each key.
  int* sl_kcnt;
  int* sl_koff;
  int* sl_bsum;
  int* sl_tr;
  int64_t sl_nk;
  // Keys with more than kKeyMaxEntries entries (attention sinks): sl_long[0]
  // counts them, sl_long[1 ..] lists their ids (at most sl_long_cap).
  int* sl_long;
  int sl_long_cap;

  float scale;
  int causal, window_left, norm;
  int grad_f32;          // dq/dk/dv element type is float32 (else the input type)
  int* dev_status;       // first device-side error, see DeviceError
};

// Key id of a support-list entry (see AttnParams::sl_kcnt): key is the K/V
// token the forward stored, b the sequence of the row (0 for varlen).
__device__ __forceinline__ int64_t list_kid(const AttnParams& p, int b, int kvh, int key) {
  return p.cu_k != nullptr ? (int64_t)kvh * p.rows_k + key : ((int64_t)b * p.hkv + kvh) * p.len_k + key;
}

// Key count of sequence b in the paged and lens_only layouts, clamped to the
// declared maximum len_k: a larger entry would index past the sequence's
// block-table row and past its per-row scratch.  A clamped length records
// kDevBadLength in the device status word.
__device__ __forceinline__ int seq_len_k(const AttnParams& p, int b) {
  const int L = p.seq_lens[b];
  if (L >= 0 && L <= p.len_k) return L;
  if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevBadLength);
  return L < 0 ? 0 : p.len_k;
}

__device__ __forceinline__ Geometry geometry(const AttnParams& p, int b) {
  Geometry g;
  if (p.cu_q != nullptr) {
    g.q_start = p.cu_q[b];
    g.q_len = p.cu_q[b + 1] - g.q_start;
    g.k_start = p.cu_k[b];
    g.k_len = p.cu_k[b + 1] - g.k_start;
  } else {
    g.q_start = b * p.len_q;
    g.q_len = p.len_q;
    g.k_start = 0;
    g.k_len = (p.paged || p.lens_only) ? seq_len_k(p, b) : p.len_k;
  }
  g.shift = p.causal_top_left ? 0 : g.k_len - g.q_len;
  return g;
}

// Element offset of query-side row i (q, o, do, dq share the indexing scheme).
__device__ __forceinline__ int64_t qrow_off(const AttnParams& p, const Geometry& g, int b, int h,
                                            int i, int64_t sb, int64_t sh, int64_t st) {
  int64_t tok = p.cu_q != nullptr ? (int64_t)(g.q_start + i) : (int64_t)i;
  return (int64_t)b * sb + (int64_t)h * sh + tok * st;
}

// Token index of key j of sequence b inside the K/V storage.  For the paged
// layout this is the physical cache row; -1 flags a page id outside the
// cache (recorded in the device status word, the row reads as zeros).
__device__ __forceinline__ int64_t key_token(const AttnParams& p, const Geometry& g, int b, int j) {
  if (p.paged) {
    int page = p.block_table[(int64_t)b * p.max_blocks + j / p.page_size];
    int64_t tok = (int64_t)page * p.page_size + (j % p.page_size);
    if (page < 0 || tok >= p.num_cache_tokens) {
      if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevBadPage);
      return -1;
    }
    return tok;
  }
  return p.cu_k != nullptr ? (int64_t)(g.k_start + j) : (int64_t)j;
}

__device__ __forceinline__ int64_t key_off(const AttnParams& p, int b, int kvh, int64_t tok,
                                           int64_t sb, int64_t sh, int64_t st) {
  // Paged caches and packed varlen tensors have no batch stride.
  int64_t bo = (p.paged || p.cu_k != nullptr) ? 0 : (int64_t)b * sb;
  return bo + (int64_t)kvh * sh + tok * st;
}

__device__ __forceinline__ int64_t stat_index(const AttnParams& p, const Geometry& g, int h, int i) {
  return (int64_t)h * p.rows_total + g.q_start + i;
}

}  // namespace hfan
