// Split-KV paged decode (one query token per sequence) for 16-bit caches.
//
// The KV cache is token-major [pages * page_size, Hkv, D]; one (token, KV
// head) row is D contiguous 16-bit values.  Work unit = (sequence, KV head,
// split of kChunk keys); each unit serves all G = Hq / Hkv query heads of the
// group, so every K/V byte is read once per group.  A row is read with one
// 16-byte load per lane by a group of D/8 lanes (coalesced 256-byte rows for
// D = 128); the dot products reduce inside the lane group with shuffles.
//
// softmax1 (2 launches):
//   split    per unit: online max / sum over its keys (no sink), partial
//            acc = sum_j 2^(s_j - m) v_j, stored with (m, l) in the workspace
//   combine  per (sequence, query head): merge the splits and add the
//            implicit zero logit once: O = sum_s 2^(m_s - M) acc_s / L,
//            L = sum_s 2^(m_s - M) l_s + 2^(-M), M = max(0, max_s m_s)
//            (reference kernels/paged_softmax1_hopper.py:17-83 semantics)
// sparsemax / entmax15 (4 launches):
//   scores   per unit: z = s * zs for every key -> workspace rows [B, Hq, max_len]
//   tau      per (sequence, query head): the row (<= 32K keys) is staged in
//            shared memory and tau is solved exactly (bracket + closed form,
//            common.cuh)
//   pv       per unit: p = (z - tau)_+^a; V rows are read only for keys with
//            p > 0 for some head of the group (zero-probability keys cost no
//            V traffic)
//   combine  O = sum over splits of the partial P V
//
// Row statistics use the same layout as the other attention kernels, so the
// general paged backward can consume them.
#include <mutex>

#include "common.cuh"
#include "params.cuh"

namespace hfan {
namespace {

constexpr int kChunk = 1024;   // keys per split
constexpr int kUnroll = 4;      // key rows in flight per lane group
constexpr int kMaxRow = 32768; // tau kernel stages at most this many keys per row

struct DecodeWs {
  float* acc;     // [B, Hkv, splits, G, D]
  float* ml;      // [B, Hkv, splits, G, 2]
  float* scores;  // [B, Hq, max_len]   (sparse only)
  float* tau;     // [B, Hq]            (sparse only)
  int splits;
};

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&x)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(src);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f32<T>(e[i]);
}
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float (&x)[8]) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f32<T>(e[i]);
}
__device__ __forceinline__ uint4 ldg16(const void* src) {
  return __ldg(reinterpret_cast<const uint4*>(src));
}

// Lane-group geometry: LPT lanes per key row (D / 8), TPW rows per warp.
template <int D>
struct Lanes {
  static constexpr int LPT = D / 8;
  static constexpr int TPW = 32 / LPT;
};

template <int LPT>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPT / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ const int* page_row(const AttnParams& p, int b) {
  return p.block_table + (int64_t)b * p.max_blocks;
}

__device__ __forceinline__ int64_t phys_token(const AttnParams& p, const int* bt, int t) {
  const int page = bt[t / p.page_size];
  const int64_t tok = (int64_t)page * p.page_size + (t % p.page_size);
  if (page < 0 || tok >= p.num_cache_tokens) {
    if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevBadPage);
    return -1;
  }
  return tok;
}

// ------------------------------------------------------------------ softmax1
// One CTA per (sequence, split) and one warp per KV head, so the 8 heads of a
// token -- one contiguous 2 KB stretch of the page -- are read together.
template <typename T, int D, int G>
__global__ void __launch_bounds__(256, 2) decode_sm1_split(AttnParams p, DecodeWs ws) {
  using LN = Lanes<D>;
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = p.seq_lens[b];
  const int t0 = split * kChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int sub = lane / LN::LPT, li = lane % LN::LPT;
  const int* bt = page_row(p, b);
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);
  const float zs = p.scale * kLog2e;
  for (int kvh = warp; kvh < p.hkv; kvh += nwarps) {
    float q[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const T* qr = static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)(kvh * G + h) * p.q_sh;
      load8<T>(qr + li * 8, q[h]);
#pragma unroll
      for (int i = 0; i < 8; ++i) q[h][i] *= zs;
    }
    float m[G], l[G], acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      m[h] = kNegInf;
      l[h] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[h][i] = 0.f;
    }
    // Warp-uniform loop bound (the group reductions are full-warp shuffles);
    // kUnroll rows per lane group are fetched before any of them is used.
    for (int tb = t0; tb < t1; tb += LN::TPW * kUnroll) {
      uint4 kr[kUnroll], vr[kUnroll];
      bool valid[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = tb + u * LN::TPW + sub;
        const int64_t tok = t < t1 ? phys_token(p, bt, t) : -1;
        valid[u] = tok >= 0;
        if (valid[u]) {
          kr[u] = ldg16(kp + tok * p.k_st + (int64_t)kvh * p.k_sh + li * 8);
          vr[u] = ldg16(vp + tok * p.v_st + (int64_t)kvh * p.v_sh + li * 8);
        } else {
          kr[u] = vr[u] = make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        float kx[8], vx[8];
        unpack8<T>(kr[u], kx);
        unpack8<T>(vr[u], vx);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float sc = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) sc = fmaf(q[h][i], kx[i], sc);
          sc = group_sum<LN::LPT>(sc);
          if (!valid[u]) continue;
          if (sc > m[h]) {
            const float a = exp2f(m[h] - sc);  // 0 on the first key
            l[h] *= a;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[h][i] *= a;
            m[h] = sc;
          }
          const float e = exp2f(sc - m[h]);
          l[h] += e;
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[h][i] = fmaf(e, vx[i], acc[h][i]);
        }
      }
    }
    // merge the lane groups of the warp (same dims, different keys)
#pragma unroll
    for (int o = LN::LPT; o < 32; o <<= 1) {
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m[h], o);
        const float l2 = __shfl_xor_sync(0xffffffffu, l[h], o);
        const float M = fmaxf(m[h], m2);
        const float f1 = m[h] > kNegInf ? exp2f(m[h] - M) : 0.f;
        const float f2 = m2 > kNegInf ? exp2f(m2 - M) : 0.f;
        l[h] = f1 * l[h] + f2 * l2;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float a2 = __shfl_xor_sync(0xffffffffu, acc[h][i], o);
          acc[h][i] = f1 * acc[h][i] + f2 * a2;
        }
        m[h] = M;
      }
    }
    if (sub == 0) {
      const int64_t unit = ((int64_t)b * p.hkv + kvh) * ws.splits + split;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float4* dst = reinterpret_cast<float4*>(ws.acc + (unit * G + h) * D + li * 8);
        dst[0] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        dst[1] = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
        if (li == 0) {
          ws.ml[(unit * G + h) * 2 + 0] = m[h];
          ws.ml[(unit * G + h) * 2 + 1] = l[h];
        }
      }
    }
  }
}

template <typename T, int D, int G>
__global__ void decode_sm1_combine(AttnParams p, DecodeWs ws) {
  const int b = blockIdx.y, hq = blockIdx.x;
  const int kvh = hq / G, h = hq % G;
  const int L = p.seq_lens[b];
  const int ns = (L + kChunk - 1) / kChunk;
  const int64_t base = ((int64_t)b * p.hkv + kvh) * ws.splits;
  float M = 0.f;  // the implicit zero logit
  for (int s = 0; s < ns; ++s) M = fmaxf(M, ws.ml[((base + s) * G + h) * 2]);
  float Lsum = exp2f(-M);
  for (int s = 0; s < ns; ++s) {
    const float ms = ws.ml[((base + s) * G + h) * 2];
    if (ms > kNegInf) Lsum = fmaf(exp2f(ms - M), ws.ml[((base + s) * G + h) * 2 + 1], Lsum);
  }
  T* orow = static_cast<T*>(p.o) + (int64_t)b * p.o_sb + (int64_t)hq * p.o_sh;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < ns; ++s) {
      const float ms = ws.ml[((base + s) * G + h) * 2];
      if (ms > kNegInf) a = fmaf(exp2f(ms - M), ws.acc[((base + s) * G + h) * D + d], a);
    }
    orow[d] = from_f32<T>(a / Lsum);
  }
  if (threadIdx.x == 0) {
    const int64_t si = (int64_t)hq * p.rows_total + b;  // len_q == 1: row index = b
    p.stats[si] = M;
    p.stats[(int64_t)p.hq * p.rows_total + si] = Lsum;
  }
}

// ------------------------------------------------------------------ sparse
template <typename T, int D, int G, int NORM>
__global__ void __launch_bounds__(256, 3) decode_sparse_scores(AttnParams p, DecodeWs ws, int max_len) {
  using LN = Lanes<D>;
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = p.seq_lens[b];
  const int t0 = split * kChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int sub = lane / LN::LPT, li = lane % LN::LPT;
  const int* bt = page_row(p, b);
  const T* kp = static_cast<const T*>(p.k);
  const float zs = NORM == HFAN_SPARSEMAX ? p.scale : 0.5f * p.scale;
  for (int kvh = warp; kvh < p.hkv; kvh += nwarps) {
    float q[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const T* qr = static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)(kvh * G + h) * p.q_sh;
      load8<T>(qr + li * 8, q[h]);
#pragma unroll
      for (int i = 0; i < 8; ++i) q[h][i] *= zs;
    }
    float* srow = ws.scores + ((int64_t)b * p.hq + kvh * G) * max_len;
    for (int tb = t0; tb < t1; tb += LN::TPW * kUnroll) {  // warp-uniform bound (shuffles)
      uint4 kr[kUnroll];
      bool valid[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = tb + u * LN::TPW + sub;
        const int64_t tok = t < t1 ? phys_token(p, bt, t) : -1;
        valid[u] = tok >= 0;
        kr[u] = valid[u] ? ldg16(kp + tok * p.k_st + (int64_t)kvh * p.k_sh + li * 8) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int t = tb + u * LN::TPW + sub;
        float kx[8];
        unpack8<T>(kr[u], kx);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          float sv = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) sv = fmaf(q[h][i], kx[i], sv);
          sv = group_sum<LN::LPT>(sv);
          if (valid[u] && li == h % LN::LPT) srow[(int64_t)h * max_len + t] = sv;
        }
      }
    }
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r += red[i];
  return r;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = kNegInf;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
  return r;
}
__device__ __forceinline__ float block_min(float v, float* red) {
  v = warp_min(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = kPosInf;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = fminf(r, red[i]);
  return r;
}

// One CTA per (sequence, query head): exact tau of the staged score row.
template <int NORM>
__global__ void __launch_bounds__(512) decode_sparse_tau(AttnParams p, DecodeWs ws, int max_len) {
  extern __shared__ float zrow[];
  __shared__ float red[32];
  const int b = blockIdx.y, hq = blockIdx.x;
  const int L = p.seq_lens[b];
  const float* srow = ws.scores + ((int64_t)b * p.hq + hq) * max_len;
  float zmax = kNegInf;
  for (int t = threadIdx.x; t < L; t += blockDim.x) {
    const float z = srow[t];
    zrow[t] = z;
    zmax = fmaxf(zmax, z);
  }
  zmax = block_max(zmax, red);
  float t = zmax - 1.f, tau = kPosInf, support = 0.f;
  if (zmax > kNegInf) {
    for (int it = 0; it < 64; ++it) {
      TauStats st{0.f, 0.f, 0.f, kPosInf};
      for (int j = threadIdx.x; j < L; j += blockDim.x) tau_accumulate(st, zrow[j], t);
      st.cnt = block_sum(st.cnt, red);
      st.s1 = block_sum(st.s1, red);
      st.s2 = block_sum(st.s2, red);
      st.zmin = block_min(st.zmin, red);
      support = st.cnt;
      if (tau_step(NORM, st, &t, &tau)) break;  // uniform: every thread sees the same sums
    }
  }
  if (threadIdx.x == 0) {
    ws.tau[(int64_t)b * p.hq + hq] = tau;
    const int64_t si = (int64_t)hq * p.rows_total + b;
    p.stats[si] = tau;
    p.stats[(int64_t)p.hq * p.rows_total + si] = support;
  }
}

template <typename T, int D, int G, int NORM>
__global__ void __launch_bounds__(256) decode_sparse_pv(AttnParams p, DecodeWs ws, int max_len) {
  using LN = Lanes<D>;
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = p.seq_lens[b];
  const int t0 = split * kChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int sub = lane / LN::LPT, li = lane % LN::LPT;
  const int* bt = page_row(p, b);
  const T* vp = static_cast<const T*>(p.v);
  for (int kvh = warp; kvh < p.hkv; kvh += nwarps) {
    float tau[G];
#pragma unroll
    for (int h = 0; h < G; ++h) tau[h] = ws.tau[(int64_t)b * p.hq + kvh * G + h];
    const float* srow = ws.scores + ((int64_t)b * p.hq + kvh * G) * max_len;
    float acc[G][8];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[h][i] = 0.f;
    for (int t = t0 + sub; t < t1; t += LN::TPW) {  // no shuffles inside: per-group bound is fine
      float pr[G];
      bool any = false;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        pr[h] = sparse_prob(NORM, srow[(int64_t)h * max_len + t], tau[h]);
        any |= pr[h] > 0.f;
      }
      if (!any) continue;
      const int64_t tok = phys_token(p, bt, t);
      if (tok < 0) continue;
      float vx[8];
      load8<T>(vp + tok * p.v_st + (int64_t)kvh * p.v_sh + li * 8, vx);
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[h][i] = fmaf(pr[h], vx[i], acc[h][i]);
    }
#pragma unroll
    for (int o = LN::LPT; o < 32; o <<= 1)
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[h][i] += __shfl_xor_sync(0xffffffffu, acc[h][i], o);
    if (sub == 0) {
      const int64_t unit = ((int64_t)b * p.hkv + kvh) * ws.splits + split;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float4* dst = reinterpret_cast<float4*>(ws.acc + (unit * G + h) * D + li * 8);
        dst[0] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
        dst[1] = make_float4(acc[h][4], acc[h][5], acc[h][6], acc[h][7]);
      }
    }
  }
}

template <typename T, int D, int G>
__global__ void decode_sparse_combine(AttnParams p, DecodeWs ws) {
  const int b = blockIdx.y, hq = blockIdx.x;
  const int kvh = hq / G, h = hq % G;
  const int ns = (p.seq_lens[b] + kChunk - 1) / kChunk;
  const int64_t base = ((int64_t)b * p.hkv + kvh) * ws.splits;
  T* orow = static_cast<T*>(p.o) + (int64_t)b * p.o_sb + (int64_t)hq * p.o_sh;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.f;
    for (int s = 0; s < ns; ++s) a += ws.acc[((base + s) * G + h) * D + d];
    orow[d] = from_f32<T>(a);
  }
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

struct WsLayout {
  size_t acc, ml, scores, tau, total;
  int splits;
};

WsLayout ws_layout(const AttnParams& p, int max_len) {
  WsLayout w;
  const int G = p.hq / p.hkv;
  w.splits = max(1, (max_len + kChunk - 1) / kChunk);
  const size_t units = (size_t)p.batch * p.hkv * w.splits;
  w.acc = 0;
  w.ml = align256(units * G * p.d * sizeof(float));
  w.scores = w.ml + align256(units * G * 2 * sizeof(float));
  if (p.norm == HFAN_SOFTMAX1) {
    w.tau = w.scores;
    w.total = w.scores;
  } else {
    w.tau = w.scores + align256((size_t)p.batch * p.hq * max_len * sizeof(float));
    w.total = w.tau + align256((size_t)p.batch * p.hq * sizeof(float));
  }
  return w;
}

template <typename T, int D, int G>
cudaError_t run(const AttnParams& p, int max_len, void* workspace, cudaStream_t s) {
  const WsLayout w = ws_layout(p, max_len);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  DecodeWs ws{reinterpret_cast<float*>(base + w.acc), reinterpret_cast<float*>(base + w.ml),
              reinterpret_cast<float*>(base + w.scores), reinterpret_cast<float*>(base + w.tau), w.splits};
  dim3 grid_u(w.splits, p.batch), grid_r(p.hq, p.batch);
  const int ut = 32 * min(p.hkv, 8);  // one warp per KV head
  if (p.norm == HFAN_SOFTMAX1) {
    decode_sm1_split<T, D, G><<<grid_u, ut, 0, s>>>(p, ws);
    decode_sm1_combine<T, D, G><<<grid_r, D, 0, s>>>(p, ws);
    return cudaGetLastError();
  }
  const size_t tau_smem = (size_t)max_len * sizeof(float);
  cudaError_t e;
  if (p.norm == HFAN_SPARSEMAX) {
    e = cudaFuncSetAttribute(decode_sparse_tau<HFAN_SPARSEMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tau_smem);
    if (e != cudaSuccess) return e;
    decode_sparse_scores<T, D, G, HFAN_SPARSEMAX><<<grid_u, ut, 0, s>>>(p, ws, max_len);
    decode_sparse_tau<HFAN_SPARSEMAX><<<grid_r, 512, tau_smem, s>>>(p, ws, max_len);
    decode_sparse_pv<T, D, G, HFAN_SPARSEMAX><<<grid_u, ut, 0, s>>>(p, ws, max_len);
  } else {
    e = cudaFuncSetAttribute(decode_sparse_tau<HFAN_ENTMAX15>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tau_smem);
    if (e != cudaSuccess) return e;
    decode_sparse_scores<T, D, G, HFAN_ENTMAX15><<<grid_u, ut, 0, s>>>(p, ws, max_len);
    decode_sparse_tau<HFAN_ENTMAX15><<<grid_r, 512, tau_smem, s>>>(p, ws, max_len);
    decode_sparse_pv<T, D, G, HFAN_ENTMAX15><<<grid_u, ut, 0, s>>>(p, ws, max_len);
  }
  decode_sparse_combine<T, D, G><<<grid_r, D, 0, s>>>(p, ws);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t run_g(const AttnParams& p, int max_len, void* ws, cudaStream_t s) {
  switch (p.hq / p.hkv) {
    case 1: return run<T, D, 1>(p, max_len, ws, s);
    case 2: return run<T, D, 2>(p, max_len, ws, s);
    case 4: return run<T, D, 4>(p, max_len, ws, s);
    default: return run<T, D, 8>(p, max_len, ws, s);
  }
}

}  // namespace

// Shapes the split-KV decode kernels serve: one query token, 16-bit cache,
// head_dim 64 or 128, up to 8 query heads per KV head, rows of at most 32K keys,
// 16-byte aligned rows.
bool decode_supported(int dtype, const AttnParams& p, int max_len) {
  if (dtype != HFAN_BFLOAT16 && dtype != HFAN_FLOAT16) return false;
  if (p.len_q != 1) return false;
  if (p.d != 64 && p.d != 128) return false;
  const int g = p.hq / p.hkv;
  if (g != 1 && g != 2 && g != 4 && g != 8) return false;
  if (max_len > kMaxRow) return false;
  auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (!al(p.q) || !al(p.k) || !al(p.v)) return false;
  if ((p.k_st % 8) || (p.k_sh % 8) || (p.v_st % 8) || (p.v_sh % 8) || (p.q_sh % 8) || (p.q_sb % 8)) return false;
  return true;
}

size_t decode_workspace_bytes(const AttnParams& p, int max_len) { return ws_layout(p, max_len).total; }

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory at the
// point where they decode: code running inside a CUDA graph capture or on an
// inference server's hot path, and embedders that own the GPU allocator and
// forbid allocations behind their back.  For them the scratch lives in this
// fixed device array instead of a caller workspace.  It is loaded with the
// library and held by every GPU that loads it until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kStaticDecodeScratchBytes = (size_t)64 << 20;  // 64 MiB
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticDecodeScratchBytes];

size_t decode_static_scratch_bytes() { return kStaticDecodeScratchBytes; }

// Device address of g_decode_scratch for the current device.  In host code the
// array name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
cudaError_t decode_static_scratch(void** out) {
  static std::mutex mu;
  static void* cache[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_scratch);
    if (e != cudaSuccess) return e;
    cache[dev] = ptr;
  }
  *out = cache[dev];
  return cudaSuccess;
}

cudaError_t decode_run(int dtype, const AttnParams& p, int max_len, void* ws, cudaStream_t s) {
  if (dtype == HFAN_BFLOAT16)
    return p.d == 128 ? run_g<__nv_bfloat16, 128>(p, max_len, ws, s) : run_g<__nv_bfloat16, 64>(p, max_len, ws, s);
  return p.d == 128 ? run_g<__half, 128>(p, max_len, ws, s) : run_g<__half, 64>(p, max_len, ws, s);
}

}  // namespace hfan
