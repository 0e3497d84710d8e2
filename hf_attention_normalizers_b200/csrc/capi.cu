// C ABI entry points (include/hfan.h): argument validation, parameter
// packing, kernel selection and error reporting.
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "params.cuh"

namespace hfan {
cudaError_t simt_attention_fwd(int dtype, const AttnParams& p, int max_q, cudaStream_t s);
cudaError_t simt_attention_bwd(int dtype, const AttnParams& p, int max_q, int max_k, cudaStream_t s);
cudaError_t rownorm_fwd(int norm, int dtype, int64_t rows, int64_t n, const void* x, int64_t ldx,
                        void* y, int64_t ldy, cudaStream_t s);
cudaError_t rownorm_bwd(int norm, int dtype, int64_t rows, int64_t n, const void* y, int64_t ldy,
                        const void* dy, int64_t lddy, void* dx, int64_t lddx, cudaStream_t s);
// Tensor-core (tcgen05 / TMA) kernels for 16-bit dense and varlen requests.
bool tc_supported(int dtype, const AttnParams& p);
// Split-KV paged decode (paged_decode.cu).
bool decode_supported(int dtype, const AttnParams& p, int max_len);
size_t decode_workspace_bytes(const AttnParams& p, int max_len);
cudaError_t decode_run(int dtype, const AttnParams& p, int max_len, void* ws, cudaStream_t s);
size_t decode_static_scratch_bytes();
cudaError_t decode_static_scratch(void** out);
cudaError_t tc_attention_fwd(int dtype, const AttnParams& p, int max_q, cudaStream_t s);
cudaError_t tc_attention_bwd(int dtype, const AttnParams& p, int max_q, int max_k, cudaStream_t s);
// Paged prefill / backward through the tensor-core kernels (paged_tc.cu);
// cudaErrorNotSupported when the shape is outside their envelope.
cudaError_t paged_tc_fwd(int dtype, const AttnParams& p, cudaStream_t s);
cudaError_t paged_tc_bwd(int dtype, const AttnParams& p, cudaStream_t s);
}  // namespace hfan

using namespace hfan;

__device__ int g_hfan_dev_status;

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(HFAN_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

// Address of the device status word on the current device: one symbol lookup
// per device, cached.
int* dev_status_ptr() {
  static std::mutex mu;
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_hfan_dev_status) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(ptr);
  }
  return cache[dev];
}

bool valid_dtype(int d) { return d == HFAN_FLOAT32 || d == HFAN_FLOAT16 || d == HFAN_BFLOAT16; }
bool valid_norm(int n) { return n == HFAN_SOFTMAX1 || n == HFAN_SPARSEMAX || n == HFAN_ENTMAX15; }

int check_common(int dtype, int norm, int batch, int hq, int hkv, int d) {
  if (!valid_dtype(dtype)) return fail(HFAN_ERR_INVALID, "unknown dtype %d", dtype);
  if (!valid_norm(norm)) return fail(HFAN_ERR_INVALID, "unknown normalizer %d", norm);
  if (batch < 1) return fail(HFAN_ERR_INVALID, "batch must be positive (got %d)", batch);
  if (hq < 1 || hkv < 1 || hq % hkv != 0)
    return fail(HFAN_ERR_INVALID, "Query heads must be divisible by KV heads (got %d and %d).", hq, hkv);
  if (d < 1 || d > 256) return fail(HFAN_ERR_INVALID, "head_dim larger than 256 is not supported.");
  return HFAN_OK;
}

void set_tensor(const hfan_tensor& t, const void** data, int64_t* sb, int64_t* sh, int64_t* st) {
  *data = t.data;
  *sb = t.stride_batch;
  *sh = t.stride_head;
  *st = t.stride_token;
}
void set_tensor(const hfan_tensor& t, void** data, int64_t* sb, int64_t* sh, int64_t* st) {
  *data = t.data;
  *sb = t.stride_batch;
  *sh = t.stride_head;
  *st = t.stride_token;
}

AttnParams base_params(const hfan_tensor& q, const hfan_tensor& k, const hfan_tensor& v,
                       const hfan_tensor& o) {
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  set_tensor(q, &p.q, &p.q_sb, &p.q_sh, &p.q_st);
  set_tensor(k, &p.k, &p.k_sb, &p.k_sh, &p.k_st);
  set_tensor(v, &p.v, &p.v_sb, &p.v_sh, &p.v_st);
  set_tensor(o, &p.o, &p.o_sb, &p.o_sh, &p.o_st);
  p.dev_status = dev_status_ptr();
  return p;
}

void set_grads(AttnParams& p, const hfan_tensor& d_o, const hfan_tensor& dq, const hfan_tensor& dk,
               const hfan_tensor& dv) {
  set_tensor(d_o, &p.dout, &p.do_sb, &p.do_sh, &p.do_st);
  set_tensor(dq, &p.dq, &p.dq_sb, &p.dq_sh, &p.dq_st);
  set_tensor(dk, &p.dk, &p.dk_sb, &p.dk_sh, &p.dk_st);
  set_tensor(dv, &p.dv, &p.dv_sb, &p.dv_sh, &p.dv_st);
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Words of the key-tile support mask (0: the request takes none).
int64_t mask_words(const hfan_attn_desc& d) {
  if (d.normalizer == HFAN_SOFTMAX1 || d.len_q <= 0 || d.len_k <= 0) return 0;
  const int64_t tiles = ceil_div(d.len_k, 128);
  if (tiles > 32 * 32) return 0;
  return (int64_t)d.heads_q * d.batch * 2 * ceil_div(d.len_q, 128) * ((tiles + 31) / 32);
}

// Byte offsets of the support-list arrays inside the caller's workspace
// (see AttnParams::sl_ent); false when the request takes no lists.
struct SupportLayout {
  int64_t flag, cnt, ent, g, kcnt, koff, bsum, tr, lng, nk, long_cap, total;
};

bool support_layout(const hfan_attn_desc& d, SupportLayout* l) {
  // sparsemax only: entmax15's supports (about 22 keys per row on N(0, 1)
  // scores at 8192 keys, against sparsemax's 4.4) make the per-entry gathers
  // cost as much as the tile kernels, and recording them in its forward (which
  // has no key indices in its candidate buffers) costs more than they save.
  if (d.normalizer != HFAN_SPARSEMAX || d.dropout_p != 0.f) return false;
  if (d.dtype != HFAN_BFLOAT16 && d.dtype != HFAN_FLOAT16) return false;
  if (d.head_dim != 64 && d.head_dim != 128) return false;
  const int64_t rows = d.cu_seqlens_q ? (int64_t)d.total_q : (int64_t)d.batch * d.len_q;
  if (rows <= 0 || d.heads_q <= 0) return false;
  const int64_t slots = (int64_t)d.heads_q * kSupSlots * rows;
  const int64_t cnt = (int64_t)d.heads_q * (d.head_dim / 32) * rows;
  if (slots >= (int64_t)1 << 31) return false;  // slot numbers are int32
  l->nk = (int64_t)d.heads_kv * (d.cu_seqlens_q ? (int64_t)d.total_k : (int64_t)d.batch * d.len_k);
  if (l->nk <= 0 || l->nk >= ((int64_t)1 << 31)) return false;  // key ids are int32 in the long-key list
  auto up = [](int64_t x) { return (x + 255) & ~int64_t(255); };
  l->flag = 0;
  l->cnt = 256;
  l->ent = l->cnt + up(cnt * 4);
  l->g = l->ent + up(slots * 8);
  l->kcnt = l->g + up(slots * 4);
  l->koff = l->kcnt + up(l->nk * 4);
  l->bsum = l->koff + up((l->nk + 1) * 4);
  l->tr = l->bsum + up(sparse_key_blocks(l->nk) * 4);
  l->lng = l->tr + up(slots * 4);
  l->long_cap = slots / (kKeyMaxEntries + 1) + 1;  // keys that can exceed kKeyMaxEntries entries
  l->total = l->lng + up((l->long_cap + 1) * 4);
  return true;
}

int fill_attn(const hfan_attn_desc* desc, AttnParams& p) {
  if (desc == nullptr) return fail(HFAN_ERR_INVALID, "null descriptor");
  int rc = check_common(desc->dtype, desc->normalizer, desc->batch, desc->heads_q, desc->heads_kv,
                        desc->head_dim);
  if (rc != HFAN_OK) return rc;
  if (desc->len_q < 0 || desc->len_k < 0) return fail(HFAN_ERR_INVALID, "negative sequence length");
  if ((desc->cu_seqlens_q == nullptr) != (desc->cu_seqlens_k == nullptr))
    return fail(HFAN_ERR_INVALID, "cu_seqlens_q and cu_seqlens_k must both be given or both be NULL");
  p.batch = desc->batch;
  p.hq = desc->heads_q;
  p.hkv = desc->heads_kv;
  p.d = desc->head_dim;
  p.len_q = desc->len_q;
  p.len_k = desc->len_k;
  p.cu_q = desc->cu_seqlens_q;
  p.cu_k = desc->cu_seqlens_k;
  p.rows_total = desc->cu_seqlens_q ? desc->total_q : desc->batch * desc->len_q;
  p.rows_k = desc->cu_seqlens_q ? desc->total_k : desc->len_k;
  p.scale = desc->scale;
  p.causal = desc->causal ? 1 : 0;
  p.window_left = desc->window_left;
  p.norm = desc->normalizer;
  p.grad_f32 = desc->grad_dtype == HFAN_FLOAT32;
  if (desc->cu_seqlens_q && desc->total_q < 0) return fail(HFAN_ERR_INVALID, "total_q must be >= 0");
  if (desc->support != nullptr) {
    SupportLayout l;
    if (!support_layout(*desc, &l))
      return fail(HFAN_ERR_INVALID, "support workspace given for a request that takes none (see hfan_attn_support_bytes)");
    if ((reinterpret_cast<uintptr_t>(desc->support) & 255u) != 0)
      return fail(HFAN_ERR_INVALID, "support workspace must be 256-byte aligned");
    uint8_t* w = static_cast<uint8_t*>(desc->support);
    p.sl_flag = reinterpret_cast<int*>(w + l.flag);
    p.sl_cnt = reinterpret_cast<int*>(w + l.cnt);
    p.sl_ent = reinterpret_cast<int2*>(w + l.ent);
    p.sl_g = reinterpret_cast<float*>(w + l.g);
    p.sl_kcnt = reinterpret_cast<int*>(w + l.kcnt);
    p.sl_koff = reinterpret_cast<int*>(w + l.koff);
    p.sl_bsum = reinterpret_cast<int*>(w + l.bsum);
    p.sl_tr = reinterpret_cast<int*>(w + l.tr);
    p.sl_nk = l.nk;
    p.sl_long = reinterpret_cast<int*>(w + l.lng);
    p.sl_long_cap = (int)l.long_cap;
  }
  if (desc->wmean.data != nullptr && desc->normalizer != HFAN_SOFTMAX1) {
    const hfan_tensor& w = desc->wmean;
    if ((reinterpret_cast<uintptr_t>(w.data) & 15u) != 0 || w.stride_token % 8 != 0 || w.stride_head % 8 != 0 ||
        w.stride_batch % 8 != 0)
      return fail(HFAN_ERR_INVALID, "wmean must be 16-byte aligned with strides that are multiples of 8 elements");
    p.wm = desc->wmean.data;
    p.wm_sb = desc->wmean.stride_batch;
    p.wm_sh = desc->wmean.stride_head;
    p.wm_st = desc->wmean.stride_token;
  }
  if (desc->key_lengths != nullptr) {
    if (desc->cu_seqlens_q != nullptr)
      return fail(HFAN_ERR_INVALID, "key_lengths applies to the dense layout only");
    p.lens_only = 1;
    p.seq_lens = desc->key_lengths;
    p.causal_top_left = 1;
  }
  if (!(desc->dropout_p >= 0.f && desc->dropout_p < 1.f)) return fail(HFAN_ERR_INVALID, "dropout_p must be in [0, 1).");
  if (desc->dropout_p > 0.f) {
    if (desc->dropout_seed == nullptr) return fail(HFAN_ERR_INVALID, "dropout_seed is required when dropout_p > 0");
    if (desc->cu_seqlens_q != nullptr)
      return fail(HFAN_ERR_UNSUPPORTED, "fused dropout is available for the dense layout only");
    p.drop_thr24 = (uint32_t)std::ceil((double)desc->dropout_p * 16777216.0);
    if (p.drop_thr24 == 0u) p.drop_thr24 = 1u;  // p > 0 but below 2^-24: drop the words below 1
    p.drop_scale = 1.f / (1.f - desc->dropout_p);
    p.drop_seed = desc->dropout_seed;
  }
  if (desc->tile_mask != nullptr) {
    if (mask_words(*desc) == 0)
      return fail(HFAN_ERR_INVALID, "tile_mask given for a request that takes none (see hfan_attn_tile_mask_words)");
    p.tile_mask = desc->tile_mask;
    p.mask_words = (int)((ceil_div(desc->len_k, 128) + 31) / 32);
    p.mask_qb = 2 * (int)ceil_div(desc->len_q, 128);
  }
  return HFAN_OK;
}

int fill_paged(const hfan_paged_desc* desc, AttnParams& p) {
  if (desc == nullptr) return fail(HFAN_ERR_INVALID, "null descriptor");
  int rc = check_common(desc->dtype, desc->normalizer, desc->batch, desc->heads_q, desc->heads_kv,
                        desc->head_dim);
  if (rc != HFAN_OK) return rc;
  if (desc->page_size < 1) return fail(HFAN_ERR_INVALID, "block_size must be positive.");
  if (desc->block_table == nullptr || desc->seq_lens == nullptr)
    return fail(HFAN_ERR_INVALID, "block_table and sequence_lengths are required");
  if (desc->len_q < 0 || desc->max_len_k < 0) return fail(HFAN_ERR_INVALID, "negative length");
  if ((int64_t)desc->max_blocks * desc->page_size < desc->max_len_k)
    return fail(HFAN_ERR_INVALID, "block_table does not contain enough blocks for sequence_lengths.");
  p.batch = desc->batch;
  p.hq = desc->heads_q;
  p.hkv = desc->heads_kv;
  p.d = desc->head_dim;
  p.len_q = desc->len_q;
  p.len_k = desc->max_len_k;
  p.rows_total = desc->batch * desc->len_q;
  p.block_table = desc->block_table;
  p.seq_lens = desc->seq_lens;
  p.page_size = desc->page_size;
  p.max_blocks = desc->max_blocks;
  p.num_cache_tokens = desc->num_cache_tokens;
  p.paged = 1;
  p.scale = desc->scale;
  p.causal = desc->causal ? 1 : 0;
  p.window_left = 0;
  p.norm = desc->normalizer;
  p.grad_f32 = 1;
  return HFAN_OK;
}

}  // namespace

extern "C" {

const char* hfan_last_error(void) { return g_err.c_str(); }
int hfan_abi_version(void) { return HFAN_ABI_VERSION; }

int hfan_device_status(int* out, int clear, void* stream) {
  if (out == nullptr) return fail(HFAN_ERR_INVALID, "null output pointer");
  int* ptr = dev_status_ptr();
  if (ptr == nullptr) return fail(HFAN_ERR_CUDA, "device status word unavailable");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, ptr, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "hfan_device_status");
  if (clear && host != 0) {
    e = cudaMemsetAsync(ptr, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "hfan_device_status(clear)");
  }
  *out = host;
  return HFAN_OK;
}

int hfan_attn_fwd(const hfan_attn_desc* desc, hfan_tensor q, hfan_tensor k, hfan_tensor v,
                  hfan_tensor o, float* stats, void* stream) {
  AttnParams p = base_params(q, k, v, o);
  int rc = fill_attn(desc, p);
  if (rc != HFAN_OK) return rc;
  if (stats == nullptr) return fail(HFAN_ERR_INVALID, "stats buffer is required");
  p.stats = stats;
  if (desc->len_q == 0 || desc->len_k == 0 || p.rows_total == 0) return HFAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  const bool tc = tc_supported(desc->dtype, p);
  if (p.sl_flag != nullptr) {
    // lists complete until a sub-list overflows; the general kernels write none
    e = cudaMemsetAsync(p.sl_flag, tc ? 0 : 1, sizeof(int), s);
    if (e != cudaSuccess) return cuda_fail(e, "hfan_attn_fwd");
  }
  if (tc) {
    e = tc_attention_fwd(desc->dtype, p, desc->len_q, s);
  } else if (p.drop_thr24 != 0u) {
    return fail(HFAN_ERR_UNSUPPORTED, "fused dropout needs 16-bit inputs with head_dim 64 or 128");
  } else {
    // the general kernels track no support: every tile counts as live
    e = p.tile_mask ? cudaMemsetAsync(p.tile_mask, 0xff, mask_words(*desc) * 4, s) : cudaSuccess;
    if (e == cudaSuccess) e = simt_attention_fwd(desc->dtype, p, desc->len_q, s);
  }
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_attn_fwd");
}

int64_t hfan_attn_tile_mask_words(const hfan_attn_desc* desc) { return desc ? mask_words(*desc) : 0; }

int64_t hfan_attn_support_bytes(const hfan_attn_desc* desc) {
  SupportLayout l;
  return desc && support_layout(*desc, &l) ? l.total : 0;
}

int hfan_attn_bwd(const hfan_attn_desc* desc, hfan_tensor q, hfan_tensor k, hfan_tensor v,
                  hfan_tensor o, hfan_tensor d_o, const float* stats, float* corr,
                  hfan_tensor dq, hfan_tensor dk, hfan_tensor dv, void* stream) {
  AttnParams p = base_params(q, k, v, o);
  int rc = fill_attn(desc, p);
  if (rc != HFAN_OK) return rc;
  if (stats == nullptr || corr == nullptr) return fail(HFAN_ERR_INVALID, "stats and corr buffers are required");
  if (!valid_dtype(desc->grad_dtype)) return fail(HFAN_ERR_INVALID, "unknown grad dtype");
  if (desc->grad_dtype != HFAN_FLOAT32 && desc->grad_dtype != desc->dtype)
    return fail(HFAN_ERR_INVALID, "grad dtype must be float32 or the input dtype");
  set_grads(p, d_o, dq, dk, dv);
  p.stats = const_cast<float*>(stats);
  p.corr = corr;
  if (desc->len_q == 0 || desc->len_k == 0 || p.rows_total == 0) return HFAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = tc_supported(desc->dtype, p) ? tc_attention_bwd(desc->dtype, p, desc->len_q, desc->len_k, s)
                                                : cudaErrorNotSupported;
  if (e == cudaErrorNotSupported && p.drop_thr24 != 0u)
    return fail(HFAN_ERR_UNSUPPORTED, "fused dropout needs 16-bit inputs and gradients with head_dim 64 or 128");
  if (e == cudaErrorNotSupported) e = simt_attention_bwd(desc->dtype, p, desc->len_q, desc->len_k, s);
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_attn_bwd");
}

int hfan_paged_fwd(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                   hfan_tensor value_cache, hfan_tensor o, float* stats, void* stream) {
  AttnParams p = base_params(q, key_cache, value_cache, o);
  int rc = fill_paged(desc, p);
  if (rc != HFAN_OK) return rc;
  if (stats == nullptr) return fail(HFAN_ERR_INVALID, "stats buffer is required");
  p.stats = stats;
  if (desc->len_q == 0 || desc->max_len_k == 0) return HFAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = paged_tc_fwd(desc->dtype, p, s);
  if (e == cudaErrorNotSupported) e = simt_attention_fwd(desc->dtype, p, desc->len_q, s);
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_paged_fwd");
}

int hfan_paged_bwd(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                   hfan_tensor value_cache, hfan_tensor o, hfan_tensor d_o, const float* stats,
                   float* corr, hfan_tensor dq, hfan_tensor dk, hfan_tensor dv, void* stream) {
  AttnParams p = base_params(q, key_cache, value_cache, o);
  int rc = fill_paged(desc, p);
  if (rc != HFAN_OK) return rc;
  if (stats == nullptr || corr == nullptr) return fail(HFAN_ERR_INVALID, "stats and corr buffers are required");
  set_grads(p, d_o, dq, dk, dv);
  p.stats = const_cast<float*>(stats);
  p.corr = corr;
  if (desc->len_q == 0 || desc->max_len_k == 0) return HFAN_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = paged_tc_bwd(desc->dtype, p, s);
  if (e == cudaErrorNotSupported) e = simt_attention_bwd(desc->dtype, p, desc->len_q, desc->max_len_k, s);
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_paged_bwd");
}

int64_t hfan_paged_decode_workspace_bytes(const hfan_paged_desc* desc) {
  AttnParams p;
  std::memset(&p, 0, sizeof(p));
  if (fill_paged(desc, p) != HFAN_OK) return -1;
  return (int64_t)decode_workspace_bytes(p, desc->max_len_k);
}

int hfan_paged_decode(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache, hfan_tensor value_cache,
                      hfan_tensor o, float* stats, void* workspace, int64_t workspace_bytes, void* stream) {
  AttnParams p = base_params(q, key_cache, value_cache, o);
  int rc = fill_paged(desc, p);
  if (rc != HFAN_OK) return rc;
  if (stats == nullptr) return fail(HFAN_ERR_INVALID, "stats buffer is required");
  p.stats = stats;
  if (!decode_supported(desc->dtype, p, desc->max_len_k))
    return fail(HFAN_ERR_UNSUPPORTED, "paged decode: shape outside the split-KV kernel's envelope");
  const size_t need = decode_workspace_bytes(p, desc->max_len_k);
  if (workspace == nullptr || workspace_bytes < (int64_t)need)
    return fail(HFAN_ERR_INVALID, "paged decode: workspace of %zu bytes required", need);
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(HFAN_ERR_INVALID, "paged decode: workspace must be 256-byte aligned");
  if (desc->max_len_k == 0) return HFAN_OK;
  cudaError_t e = decode_run(desc->dtype, p, desc->max_len_k, workspace, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_paged_decode");
}

int hfan_paged_decode_static(const hfan_paged_desc* desc, hfan_tensor q, hfan_tensor key_cache,
                             hfan_tensor value_cache, hfan_tensor o, float* stats, void* stream) {
  AttnParams p = base_params(q, key_cache, value_cache, o);
  int rc = fill_paged(desc, p);
  if (rc != HFAN_OK) return rc;
  if (stats == nullptr) return fail(HFAN_ERR_INVALID, "stats buffer is required");
  p.stats = stats;
  if (!decode_supported(desc->dtype, p, desc->max_len_k))
    return fail(HFAN_ERR_UNSUPPORTED, "paged decode: shape outside the split-KV kernel's envelope");
  const size_t need = decode_workspace_bytes(p, desc->max_len_k);
  const size_t have = decode_static_scratch_bytes();
  if (need > have)
    return fail(HFAN_ERR_INVALID,
                "hfan_paged_decode_static: this request needs %zu bytes of scratch but the built-in "
                "scratch holds %zu bytes; use hfan_paged_decode with a caller workspace",
                need, have);
  void* ws = nullptr;
  cudaError_t e = decode_static_scratch(&ws);
  if (e != cudaSuccess) return cuda_fail(e, "hfan_paged_decode_static (scratch address)");
  if (desc->max_len_k == 0) return HFAN_OK;
  e = decode_run(desc->dtype, p, desc->max_len_k, ws, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_paged_decode_static");
}

int hfan_rownorm_fwd(int32_t normalizer, int32_t dtype, int64_t rows, int64_t n, const void* x,
                     int64_t ld_x, void* y, int64_t ld_y, void* stream) {
  if (!valid_norm(normalizer) || !valid_dtype(dtype)) return fail(HFAN_ERR_INVALID, "bad normalizer or dtype");
  if (rows < 0 || n < 0 || ld_x < n || ld_y < n) return fail(HFAN_ERR_INVALID, "bad matrix shape");
  if (rows == 0 || n == 0) return HFAN_OK;
  if (rows > (int64_t)8 * 2147483647LL) return fail(HFAN_ERR_INVALID, "too many rows");
  cudaError_t e = rownorm_fwd(normalizer, dtype, rows, n, x, ld_x, y, ld_y, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_rownorm_fwd");
}

int hfan_rownorm_bwd(int32_t normalizer, int32_t dtype, int64_t rows, int64_t n, const void* y,
                     int64_t ld_y, const void* dy, int64_t ld_dy, void* dx, int64_t ld_dx,
                     void* stream) {
  if (!valid_norm(normalizer) || !valid_dtype(dtype)) return fail(HFAN_ERR_INVALID, "bad normalizer or dtype");
  if (rows < 0 || n < 0 || ld_y < n || ld_dy < n || ld_dx < n) return fail(HFAN_ERR_INVALID, "bad matrix shape");
  if (rows == 0 || n == 0) return HFAN_OK;
  if (rows > (int64_t)8 * 2147483647LL) return fail(HFAN_ERR_INVALID, "too many rows");
  cudaError_t e = rownorm_bwd(normalizer, dtype, rows, n, y, ld_y, dy, ld_dy, dx, ld_dx,
                              static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HFAN_OK : cuda_fail(e, "hfan_rownorm_bwd");
}

}  // extern "C"
