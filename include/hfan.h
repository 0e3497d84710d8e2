/*
 * hfan.h -- C ABI of the B200 fused normalizer-attention engine.
 *
 * Plain pointers, sizes and strides only: no torch types cross this boundary.
 * Every entry point enqueues work on the caller's CUDA stream and returns an
 * hfan_status; hfan_last_error() returns a thread-local description of the
 * last failure.  Nothing here allocates device memory unless stated.
 *
 * The reference exposes this path as Python functions that launch Triton
 * kernels inside torch.autograd.Functions; each entry point below replaces the
 * kernel launches behind one of them:
 *
 *   hfan_attn_fwd / hfan_attn_bwd
 *       dense [B,H,S,D] and packed varlen [T,H,D] attention
 *       replaces _softmax1_forward_kernel / _softmax1_backward_kernel
 *         (hf_attention_normalizers/kernels/softmax1_hopper.py:20-315, launched at :335-409),
 *       _multi_block_forward_kernel / _multi_block_backward_kernel
 *         (kernels/sparse_entmax_hopper.py:30-328, launched at :337-425),
 *       varlen _forward/_backward
 *         (kernels/varlen_softmax1_hopper.py:26-149, kernels/varlen_sparse_entmax_hopper.py:22-126).
 *   hfan_paged_fwd / hfan_paged_bwd
 *       paged KV cache [pages*page_size, Hkv, D] + block_table
 *       replaces _paged_sparse_forward/_backward/_kv_backward
 *         (kernels/paged_sparse_entmax_hopper.py:52-386, launched at :395-461) and
 *       _paged_softmax1_forward/_backward/_kv_backward
 *         (kernels/paged_softmax1_hopper.py:17-278, launched at :287-349).
 *   hfan_rownorm_fwd / hfan_rownorm_bwd
 *       row-wise softmax1 / sparsemax / entmax15 on a materialised score matrix
 *       replaces the eager autograd Functions softmax_n_shifted_zeros
 *         (vutils/softmax1.py:4-21), SparsemaxFunction (vutils/entmax.py:136-157),
 *         Entmax15Function (vutils/entmax.py:160-183).
 *
 * Semantics shared by all attention entry points (same as the reference kernels):
 *   scores s = scale * q.k ; causal masks are bottom-right aligned
 *   (key j visible to query row i iff j <= i + Lk - Lq); window_left > 0 also
 *   hides keys j <= i + Lk - Lq - window_left; GQA maps query head h to KV head
 *   h / (Hq / Hkv).  A query row with no visible key yields a zero output row
 *   and zero gradients.
 */
#ifndef HFAN_H_
#define HFAN_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HFAN_ABI_VERSION 2

typedef enum hfan_status {
  HFAN_OK = 0,
  HFAN_ERR_INVALID = 1,      /* bad argument (shape, stride, alignment, range)   */
  HFAN_ERR_UNSUPPORTED = 2,  /* valid request this build has no kernel for        */
  HFAN_ERR_CUDA = 3,         /* a CUDA runtime/driver call failed                 */
  HFAN_ERR_DEVICE = 4        /* a kernel reported an error (bounded wait expired, */
                             /* out-of-range page index) through its status word  */
} hfan_status;

typedef enum hfan_normalizer {
  HFAN_SOFTMAX1 = 0,   /* exp(x_i) / (1 + sum_j exp(x_j))                      */
  HFAN_SPARSEMAX = 1,  /* Euclidean projection onto the simplex                 */
  HFAN_ENTMAX15 = 2    /* 1.5-entmax of x (computed as in vutils: z = (x-max)/2) */
} hfan_normalizer;

typedef enum hfan_dtype { HFAN_FLOAT32 = 0, HFAN_FLOAT16 = 1, HFAN_BFLOAT16 = 2 } hfan_dtype;

/* A strided [batch, head, token, dim] view.  The dim stride is 1.  Strides are
 * in elements.  Packed varlen tensors [T, H, D] use stride_batch = 0 and the
 * cu_seqlens offsets of hfan_attn_desc. */
typedef struct hfan_tensor {
  void* data;
  int64_t stride_batch;
  int64_t stride_head;
  int64_t stride_token;
} hfan_tensor;

typedef struct hfan_attn_desc {
  int32_t dtype;        /* hfan_dtype of q, k, v, o, do                               */
  int32_t normalizer;   /* hfan_normalizer                                            */
  int32_t batch;        /* number of sequences                                        */
  int32_t heads_q;
  int32_t heads_kv;     /* heads_q % heads_kv == 0                                    */
  int32_t head_dim;     /* 1..256                                                     */
  int32_t len_q;        /* dense: query length; varlen: max query length              */
  int32_t len_k;        /* dense: key length;   varlen: max key length                */
  int32_t total_q;      /* varlen: packed query tokens (rows of q); dense: ignored    */
  int32_t total_k;      /* varlen: packed key tokens (rows of k, v); dense: ignored   */
  const int32_t* cu_seqlens_q; /* varlen: [batch+1] device offsets, else NULL         */
  const int32_t* cu_seqlens_k; /* varlen: [batch+1] device offsets, else NULL         */
  float scale;
  int32_t causal;
  int32_t window_left;  /* <= 0: no window                                            */
  int32_t grad_dtype;   /* hfan_dtype of dq/dk/dv written by hfan_attn_bwd            */
  uint32_t* tile_mask;  /* sparsemax/entmax15: support bitmask of key tiles, or NULL   */
                        /* (see hfan_attn_tile_mask_words)                             */
  float dropout_p;      /* [0, 1): attention dropout; 0 = none.  Dense 16-bit inputs   */
                        /* with head_dim 64/128 only (else HFAN_ERR_UNSUPPORTED).      */
  const int64_t* dropout_seed; /* device int64 seed (required when dropout_p > 0);     */
                        /* forward and backward must get the same value.  Replaces the */
                        /* saved seed of kernels/softmax1_hopper.py:434-441.           */
  const int32_t* key_lengths; /* dense layout: [batch] device key counts (keys j <   */
                        /* key_lengths[b] exist), or NULL = len_k for every sequence.  */
                        /* With it the causal mask is aligned at the first key (row i  */
                        /* sees j <= i): HF's causal mask of a right-padded batch.     */
                        /* Replaces _hopper_right_padded_attention (backends.py:409-472) */
                        /* with one launch.  Gradients of keys past a length are not   */
                        /* written.                                                    */
  hfan_tensor wmean;    /* sparsemax/entmax15, tensor-core path: [B, Hq, S, D] (dtype  */
                        /* of q) written by the forward: per row the w-weighted mean   */
                        /* of V, sum_j w_j v_j / sum_j w_j with w = 1[p > 0]            */
                        /* (sparsemax) or sqrt(p) (entmax15).  The backward then gets  */
                        /* the row correction c = dO . wmean without a second sweep    */
                        /* over the keys.  data = NULL: not produced / not used.  No   */
                        /* counterpart in the reference (its backward sweeps twice,    */
                        /* kernels/sparse_entmax_hopper.py:230-300).                   */
  void* support;        /* sparsemax without dropout, 16-bit inputs, head_dim          */
                        /* 64/128: device workspace of hfan_attn_support_bytes(desc)   */
                        /* bytes (256-byte aligned), or NULL.  hfan_attn_fwd writes    */
                        /* every row's support list into it (the keys with p > 0, up  */
                        /* to 64 per row); hfan_attn_bwd given the same workspace     */
                        /* computes dQ, the row correction, dK and dV from the lists  */
                        /* (transposed to the keys) instead of sweeping every key     */
                        /* tile, and falls back to the tile kernels when a list       */
                        /* overflowed (or, for dK/dV, a key held by more than 524288  */
                        /* (head, row) pairs).  Results are the same on every run.    */
                        /* No counterpart in the                                       */
                        /* reference (its backward recomputes every tile,             */
                        /* kernels/sparse_entmax_hopper.py:230-319).                   */
} hfan_attn_desc;

/* Row statistics saved by the forward for the backward: float32 [2, heads_q, rows]
 * where rows = batch*len_q (dense, row = b*len_q + i) or total packed tokens
 * (varlen).  softmax1: stats[0] = running max m (log2 units, >= 0), stats[1] =
 * denominator l.  sparsemax/entmax15: stats[0] = threshold tau in z units
 * (z = s for sparsemax, z = s/2 for entmax15; +inf for an empty row),
 * stats[1] = support size.  The backward also uses a float32 [heads_q, rows]
 * scratch ("corr") for the per-row correction term. */

int hfan_attn_fwd(const hfan_attn_desc* desc, hfan_tensor q, hfan_tensor k, hfan_tensor v,
                  hfan_tensor o, float* stats, void* stream);

/* Key-tile support mask of the sparse normalizers (no counterpart in the
 * reference; its kernels sweep every key tile, kernels/sparse_entmax_hopper.py:126-151
 * and :271-319).  When desc->tile_mask is set, hfan_attn_fwd writes one bit per
 * (query head, sequence, 64-row query block, 128-key tile): set when any
 * probability of those rows on those keys is nonzero.  hfan_attn_bwd given the
 * same buffer skips the tiles whose bit is clear (all-zero probabilities
 * contribute nothing to any gradient).  Layout: uint32 words
 * [heads_q][batch][2 * ceil(len_q / 128)][W], W = ceil(ceil(len_k / 128) / 32),
 * bit t % 32 of word t / 32 = key tile t.  Returns the number of words, or 0
 * when the request takes no mask (softmax1, or rows longer than 131072 keys);
 * then desc->tile_mask must be NULL. */
int64_t hfan_attn_tile_mask_words(const hfan_attn_desc* desc);

/* Bytes of the support-list workspace for desc (see hfan_attn_desc.support), or
 * 0 when the request takes none (softmax1, entmax15, dropout, fp32 inputs,
 * other head dims).  No counterpart in the reference. */
int64_t hfan_attn_support_bytes(const hfan_attn_desc* desc);

int hfan_attn_bwd(const hfan_attn_desc* desc, hfan_tensor q, hfan_tensor k, hfan_tensor v,
                  hfan_tensor o, hfan_tensor d_o, const float* stats, float* corr,
                  hfan_tensor dq, hfan_tensor dk, hfan_tensor dv, void* stream);

typedef struct hfan_paged_desc {
  int32_t dtype;
  int32_t normalizer;
  int32_t batch;
  int32_t heads_q;
  int32_t heads_kv;
  int32_t head_dim;
  int32_t len_q;                /* query tokens per sequence (1 for decode)              */
  int32_t page_size;            /* tokens per physical page                              */
  int32_t max_blocks;           /* block_table row stride (columns)                      */
  int32_t max_len_k;            /* upper bound of seq_lens (grid sizing)                 */
  int64_t num_cache_tokens;     /* rows of key_cache / value_cache (bounds checks)       */
  const int32_t* block_table;   /* [batch, max_blocks] physical page ids                 */
  const int32_t* seq_lens;      /* [batch] key length of each sequence                   */
  float scale;
  int32_t causal;
  int32_t grad_dtype;
} hfan_paged_desc;

/* q, o, d_o, dq: [batch, heads_q, len_q, D] views.  key_cache/value_cache and
 * their gradients: stride_batch is ignored, stride_token / stride_head address
 * [num_cache_tokens, heads_kv, D].  Stats as for hfan_attn_fwd with rows =
 * batch*len_q.  dk/dv must be zero-filled float32: pages shared between
 * sequences accumulate.  16-bit caches with head_dim 64/128 and len_q > 1 run
 * on the tensor-core kernels (pages gathered into stream-ordered scratch,
 * released on `stream`); other shapes on the general kernels. */
int hfan_paged_fwd(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                   hfan_tensor value_cache, hfan_tensor o, float* stats, void* stream);

int hfan_paged_bwd(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                   hfan_tensor value_cache, hfan_tensor o, hfan_tensor d_o, const float* stats,
                   float* corr, hfan_tensor dq, hfan_tensor dk, hfan_tensor dv, void* stream);

/* Split-KV paged decode (len_q == 1), the serving fast path of hfan_paged_fwd.
 * Same semantics, inputs, outputs and statistics as hfan_paged_fwd; scratch
 * (per-split partial outputs and, for sparsemax/entmax15, the score rows) lives
 * in a caller-provided device workspace, 256-byte aligned, of at least
 * hfan_paged_decode_workspace_bytes(desc) bytes.  Returns HFAN_ERR_UNSUPPORTED
 * (nothing launched) for shapes outside the kernel's envelope: 16-bit cache,
 * head_dim 64/128, heads_q/heads_kv in {1,2,4,8}, max_len_k <= 32768.
 * Replaces _paged_softmax1_forward (kernels/paged_softmax1_hopper.py:17-83) and
 * _paged_sparse_forward (kernels/paged_sparse_entmax_hopper.py:52-185) for decode. */
int64_t hfan_paged_decode_workspace_bytes(const hfan_paged_desc* desc);
int hfan_paged_decode(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                      hfan_tensor value_cache, hfan_tensor o, float* stats, void* workspace,
                      int64_t workspace_bytes, void* stream);

/* Allocation-free paged decode.  This entry point has no counterpart in the
 * reference.  It is for callers that cannot allocate device memory when they
 * decode: code running on a serving hot path, and embedders that own the GPU
 * allocator.  It does exactly what
 * hfan_paged_decode does, but its scratch is a fixed 64 MiB device array
 * inside the library (every GPU that loads the library holds it until the
 * process exits), so the caller passes only inputs and outputs.
 *   - Requests needing more than 64 MiB of scratch (see
 *     hfan_paged_decode_workspace_bytes) fail with HFAN_ERR_INVALID and a
 *     message; nothing is launched.
 *   - The first call on a device looks up the array's device address with
 *     that device current; make that first call before any stream capture.
 *   - All calls share the one array, and it keeps the previous call's
 *     contents (every kernel overwrites the scratch it later reads, so nothing
 *     needs clearing).  Calls that overlap on the GPU (different streams, or
 *     different threads) race on it: serialise them.
 *   - The looked-up address is kept for the life of the process: do not call
 *     cudaDeviceReset on a device while this library is loaded.
 *   - Nothing here calls cudaMalloc, cudaFree or an allocating library. */
int hfan_paged_decode_static(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                             hfan_tensor value_cache, hfan_tensor o, float* stats, void* stream);

/* Row normalizers over the last axis of a [rows, n] matrix with row stride
 * ld (elements, unit column stride).  y/dx have the dtype of x. */
int hfan_rownorm_fwd(int32_t normalizer, int32_t dtype, int64_t rows, int64_t n,
                     const void* x, int64_t ld_x, void* y, int64_t ld_y, void* stream);
int hfan_rownorm_bwd(int32_t normalizer, int32_t dtype, int64_t rows, int64_t n,
                     const void* y, int64_t ld_y, const void* dy, int64_t ld_dy,
                     void* dx, int64_t ld_dx, void* stream);

/* Synchronises `stream`, then reads the device status word of the current
 * device (0 = no error, 1 = out-of-range page id, 2 = bounded wait expired,
 * 3 = a sequence_lengths entry outside [0, max_len_k], clamped into that range)
 * into *out; clear != 0 resets it. */
int hfan_device_status(int* out, int clear, void* stream);

/* Thread-local message for the last non-OK status of this thread. */
const char* hfan_last_error(void);
int hfan_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* HFAN_H_ */
