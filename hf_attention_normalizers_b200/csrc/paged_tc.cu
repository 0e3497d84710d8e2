// Paged prefill and backward on the tensor-core kernels.
//
// The pages of every sequence are gathered (16-byte copies) into a dense,
// zero-padded [B, Hkv, max_len_k, D] buffer; the dense tensor-core kernels run
// on it with per-sequence key lengths (AttnParams::lens_only: geometry reads
// seq_lens, K/V are addressed densely); the backward scatters dK / dV back
// into the caller's float32 page gradients with atomic adds (pages may be
// shared between sequences) and widens dQ to float32.  Scratch comes from the
// stream-ordered allocator and is released on the same stream.
#include "common.cuh"
#include "params.cuh"

namespace hfan {

bool tc_supported(int dtype, const AttnParams& p);
cudaError_t tc_attention_fwd(int dtype, const AttnParams& p, int max_q, cudaStream_t s);
cudaError_t tc_attention_bwd(int dtype, const AttnParams& p, int max_q, int max_k, cudaStream_t s);

namespace {

// Physical cache row of token t of sequence b, or -1 (page id out of range).
__device__ __forceinline__ int64_t cache_row(const AttnParams& p, int b, int t) {
  const int page = p.block_table[(int64_t)b * p.max_blocks + t / p.page_size];
  const int64_t row = (int64_t)page * p.page_size + (t % p.page_size);
  if (page < 0 || row >= p.num_cache_tokens) {
    if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevBadPage);
    return -1;
  }
  return row;
}

// One thread per 16-byte chunk of a (sequence, head, token) row; tokens past
// the sequence (and rows of invalid pages) are zero.
__global__ void gather_pages(AttnParams p, uint4* kd, uint4* vd, int lmax) {
  const int chunks = p.d / 8;
  const int64_t n = (int64_t)p.batch * p.hkv * lmax * chunks;
  for (int64_t x = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; x < n; x += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(x % chunks);
    const int t = (int)((x / chunks) % lmax);
    const int h = (int)((x / ((int64_t)chunks * lmax)) % p.hkv);
    const int b = (int)(x / ((int64_t)chunks * lmax * p.hkv));
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (t < seq_len_k(p, b)) {
      const int64_t row = cache_row(p, b, t);
      if (row >= 0) {
        const uint16_t* kc = static_cast<const uint16_t*>(p.k);
        const uint16_t* vc = static_cast<const uint16_t*>(p.v);
        kv = *reinterpret_cast<const uint4*>(kc + row * p.k_st + (int64_t)h * p.k_sh + c * 8);
        vv = *reinterpret_cast<const uint4*>(vc + row * p.v_st + (int64_t)h * p.v_sh + c * 8);
      }
    }
    kd[x] = kv;
    vd[x] = vv;
  }
}

// dK / dV of the dense buffer -> float32 page gradients (atomic adds).
template <typename T>
__global__ void scatter_grads(AttnParams p, const T* dkd, const T* dvd, int lmax) {
  const int64_t n = (int64_t)p.batch * p.hkv * lmax * p.d;
  float* dk = static_cast<float*>(p.dk);
  float* dv = static_cast<float*>(p.dv);
  for (int64_t x = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; x < n; x += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)(x % p.d);
    const int t = (int)((x / p.d) % lmax);
    const int h = (int)((x / ((int64_t)p.d * lmax)) % p.hkv);
    const int b = (int)(x / ((int64_t)p.d * lmax * p.hkv));
    if (t >= seq_len_k(p, b)) continue;
    const int64_t row = cache_row(p, b, t);
    if (row < 0) continue;
    atomicAdd(dk + row * p.dk_st + (int64_t)h * p.dk_sh + e, to_f32<T>(dkd[x]));
    atomicAdd(dv + row * p.dv_st + (int64_t)h * p.dv_sh + e, to_f32<T>(dvd[x]));
  }
}

// dQ of the dense [B, Hq, Lq, D] buffer -> the caller's float32 dq.
template <typename T>
__global__ void widen_dq(AttnParams p, const T* src) {
  const int64_t n = (int64_t)p.batch * p.hq * p.len_q * p.d;
  float* dq = static_cast<float*>(p.dq);
  for (int64_t x = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; x < n; x += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)(x % p.d);
    const int i = (int)((x / p.d) % p.len_q);
    const int h = (int)((x / ((int64_t)p.d * p.len_q)) % p.hq);
    const int b = (int)(x / ((int64_t)p.d * p.len_q * p.hq));
    dq[(int64_t)b * p.dq_sb + (int64_t)h * p.dq_sh + (int64_t)i * p.dq_st + e] = to_f32<T>(src[x]);
  }
}

int grid_for(int64_t n) {
  const int64_t blocks = (n + 255) / 256;
  return (int)(blocks < 148 * 32 ? blocks : 148 * 32);
}

// The dense view of the gathered buffers (K/V [B, Hkv, lmax, D] contiguous),
// or false when the tensor-core kernels do not serve the shape.
bool dense_view(int dtype, const AttnParams& p, const void* kd, const void* vd, int lmax, AttnParams* out) {
  AttnParams d = p;
  d.paged = 0;
  d.lens_only = 1;
  d.k = kd;
  d.v = vd;
  d.k_st = d.v_st = p.d;
  d.k_sh = d.v_sh = (int64_t)lmax * p.d;
  d.k_sb = d.v_sb = (int64_t)p.hkv * lmax * p.d;
  d.len_k = lmax;
  *out = d;
  return tc_supported(dtype, d);
}

// Shapes and dtypes the route serves (checked before anything is allocated).
bool route_ok(int dtype, const AttnParams& p) {
  if (dtype != HFAN_BFLOAT16 && dtype != HFAN_FLOAT16) return false;
  if (p.d != 64 && p.d != 128) return false;
  if (p.len_q < 2 || p.len_k < 1) return false;  // len_q == 1 is the split-KV decode's
  if ((p.k_st % 8) || (p.k_sh % 8) || (p.v_st % 8) || (p.v_sh % 8)) return false;
  if ((reinterpret_cast<uintptr_t>(p.k) & 15) || (reinterpret_cast<uintptr_t>(p.v) & 15)) return false;
  AttnParams probe;  // (the gathered buffers come from the allocator: 256-byte aligned)
  const void* aligned = reinterpret_cast<const void*>(uintptr_t(256));
  return dense_view(dtype, p, aligned, aligned, p.len_k, &probe);
}

}  // namespace

cudaError_t paged_tc_fwd(int dtype, const AttnParams& p, cudaStream_t s) {
  if (!route_ok(dtype, p)) return cudaErrorNotSupported;
  const int lmax = p.len_k;
  const size_t bytes = (size_t)p.batch * p.hkv * lmax * p.d * 2;
  void *kd = nullptr, *vd = nullptr;
  cudaError_t e = cudaMallocAsync(&kd, bytes, s);
  if (e != cudaSuccess) return e;
  e = cudaMallocAsync(&vd, bytes, s);
  if (e == cudaSuccess) {
    gather_pages<<<grid_for((int64_t)bytes / 16), 256, 0, s>>>(p, static_cast<uint4*>(kd), static_cast<uint4*>(vd),
                                                                lmax);
    e = cudaGetLastError();
    AttnParams d;
    if (e == cudaSuccess) e = dense_view(dtype, p, kd, vd, lmax, &d) ? tc_attention_fwd(dtype, d, p.len_q, s)
                                                                      : cudaErrorNotSupported;
    cudaFreeAsync(vd, s);
  }
  cudaFreeAsync(kd, s);
  return e;
}

cudaError_t paged_tc_bwd(int dtype, const AttnParams& p, cudaStream_t s) {
  if (!route_ok(dtype, p)) return cudaErrorNotSupported;
  const int lmax = p.len_k;
  const size_t kv_bytes = (size_t)p.batch * p.hkv * lmax * p.d * 2;
  const size_t q_bytes = (size_t)p.batch * p.hq * p.len_q * p.d * 2;
  // one allocation: K, V, dK, dV (dense, kv_bytes each) and dQ (q_bytes)
  char* buf = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&buf), 4 * kv_bytes + q_bytes, s);
  if (e != cudaSuccess) return e;
  void *kd = buf, *vd = buf + kv_bytes, *dkd = buf + 2 * kv_bytes, *dvd = buf + 3 * kv_bytes,
       *dqd = buf + 4 * kv_bytes;
  gather_pages<<<grid_for((int64_t)kv_bytes / 16), 256, 0, s>>>(p, static_cast<uint4*>(kd), static_cast<uint4*>(vd),
                                                                lmax);
  e = cudaGetLastError();
  AttnParams d;
  if (e == cudaSuccess && !dense_view(dtype, p, kd, vd, lmax, &d)) e = cudaErrorNotSupported;
  if (e == cudaSuccess) {
    d.grad_f32 = 0;
    d.dq = dqd;
    d.dq_st = p.d;
    d.dq_sh = (int64_t)p.len_q * p.d;
    d.dq_sb = (int64_t)p.hq * p.len_q * p.d;
    d.dk = dkd;
    d.dv = dvd;
    d.dk_st = d.dv_st = p.d;
    d.dk_sh = d.dv_sh = (int64_t)lmax * p.d;
    d.dk_sb = d.dv_sb = (int64_t)p.hkv * lmax * p.d;
    e = tc_attention_bwd(dtype, d, p.len_q, lmax, s);
  }
  if (e == cudaSuccess) {
    const int64_t nkv = (int64_t)p.batch * p.hkv * lmax * p.d, nq = (int64_t)p.batch * p.hq * p.len_q * p.d;
    if (dtype == HFAN_BFLOAT16) {
      scatter_grads<__nv_bfloat16><<<grid_for(nkv), 256, 0, s>>>(p, static_cast<const __nv_bfloat16*>(dkd),
                                                                 static_cast<const __nv_bfloat16*>(dvd), lmax);
      widen_dq<__nv_bfloat16><<<grid_for(nq), 256, 0, s>>>(p, static_cast<const __nv_bfloat16*>(dqd));
    } else {
      scatter_grads<__half><<<grid_for(nkv), 256, 0, s>>>(p, static_cast<const __half*>(dkd),
                                                          static_cast<const __half*>(dvd), lmax);
      widen_dq<__half><<<grid_for(nq), 256, 0, s>>>(p, static_cast<const __half*>(dqd));
    }
    e = cudaGetLastError();
  }
  cudaFreeAsync(buf, s);
  return e;
}

}  // namespace hfan
