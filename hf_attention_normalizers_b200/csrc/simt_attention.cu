// General-purpose fused attention kernels on CUDA cores (fp32 arithmetic).
//
// These serve the requests the tensor-core kernels do not take: float32
// inputs (the 1e-5 parity bar needs fp32 products), head dims that are not a
// multiple of 64, and the paged layout with more than one query token.  They
// keep the reference's semantics (kernels/softmax1_hopper.py,
// kernels/sparse_entmax_hopper.py, the varlen and paged kernels) but solve the
// sparse threshold exactly instead of by 24 bisection sweeps.
//
// Forward / dQ kernels: one warp per query row, 8 rows per CTA, keys in tiles
// of 32 staged in shared memory as fp32; lane l scores key (tile + l).
// dK/dV kernel: one warp per key, 8 keys per CTA, query rows in tiles of 32;
// each CTA walks every query head of its KV group, so GQA needs no atomics.
// Paged dK/dV accumulate with atomics because pages may be shared.
#include "common.cuh"
#include "params.cuh"

namespace hfan {

constexpr int kRows = 8;   // warps (query rows or keys) per CTA
constexpr int kTile = 32;  // keys (or query rows) per shared-memory tile
constexpr int kMaxDimRegs = 8;  // head_dim <= 256 -> 8 dims per lane

template <int NORM> __device__ __forceinline__ float zscale_of(float scale) {
  return NORM == HFAN_SOFTMAX1 ? scale * kLog2e : (NORM == HFAN_SPARSEMAX ? scale : 0.5f * scale);
}

// Stage keys [kb, kb+32) of (b, kvh) from `src` into dst[32][ld] as fp32.
template <typename T>
__device__ __forceinline__ void load_key_tile(const AttnParams& p, const Geometry& g, int b,
                                              int kvh, int kb, int k_hi, const T* src,
                                              int64_t sb, int64_t sh, int64_t st, float* dst,
                                              int ld) {
  const int D = p.d;
  for (int idx = threadIdx.x; idx < kTile * D; idx += blockDim.x) {
    int r = idx / D, c = idx - r * D;
    int j = kb + r;
    float val = 0.f;
    if (j < k_hi) {
      int64_t tok = key_token(p, g, b, j);
      if (tok >= 0) val = to_f32<T>(src[key_off(p, b, kvh, tok, sb, sh, st) + c]);
    }
    dst[r * ld + c] = val;
  }
}

__device__ __forceinline__ float dot_row(const float* a, const float* bvec, int D) {
  float acc = 0.f;
#pragma unroll 4
  for (int d = 0; d < D; ++d) acc = fmaf(a[d], bvec[d], acc);
  return acc;
}

// --------------------------------------------------------------------------
// Forward
// --------------------------------------------------------------------------
template <typename T, int NORM>
__global__ void __launch_bounds__(kRows * 32) simt_fwd_kernel(AttnParams p) {
  extern __shared__ float smem[];
  const int D = p.d, Dp = D + 1;
  float* Ks = smem;               // [32][Dp]
  float* Vs = Ks + kTile * Dp;    // [32][Dp]
  float* Qs = Vs + kTile * Dp;    // [8][D]
  const int b = blockIdx.z, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Geometry g = geometry(p, b);
  const int q0 = blockIdx.x * kRows;
  if (q0 >= g.q_len) return;
  const int row = q0 + warp;
  const bool active = row < g.q_len;
  const int kvh = h / (p.hq / p.hkv);
  const T* qp = static_cast<const T*>(p.q);
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);

  for (int d = lane; d < D; d += 32)
    Qs[warp * D + d] = active ? to_f32<T>(qp[qrow_off(p, g, b, h, row, p.q_sb, p.q_sh, p.q_st) + d]) : 0.f;

  const int last_row = min(q0 + kRows - 1, g.q_len - 1);
  int k_hi = g.k_len;
  if (p.causal) k_hi = min(k_hi, last_row + g.shift + 1);
  int k_lo = 0;
  if (p.window_left > 0) k_lo = max(0, q0 + g.shift - p.window_left + 1);
  k_lo = (k_lo / kTile) * kTile;
  const float zs = zscale_of<NORM>(p.scale);

  auto score = [&](int kb) -> float {
    int j = kb + lane;
    float s = dot_row(Qs + warp * D, Ks + lane * Dp, D);
    return (active && key_visible(row, j, g, p.causal, p.window_left)) ? s * zs : kNegInf;
  };

  float acc[kMaxDimRegs];
#pragma unroll
  for (int i = 0; i < kMaxDimRegs; ++i) acc[i] = 0.f;
  auto accumulate_pv = [&](float pj) {
    for (int jj = 0; jj < kTile; ++jj) {
      float pr = __shfl_sync(0xffffffffu, pj, jj);
      if (pr != 0.f) {
#pragma unroll
        for (int i = 0; i < kMaxDimRegs; ++i) {
          int d = lane + 32 * i;
          if (d < D) acc[i] = fmaf(pr, Vs[jj * Dp + d], acc[i]);
        }
      }
    }
  };

  float stat0, stat1;
  if (NORM == HFAN_SOFTMAX1) {
    // Online max / denominator seeded with the implicit zero logit (m = 0,
    // l = 1), as kernels/softmax1_hopper.py:80-83; log2 units.
    float m = 0.f, l = 1.f;
    for (int kb = k_lo; kb < k_hi; kb += kTile) {
      __syncthreads();
      load_key_tile<T>(p, g, b, kvh, kb, k_hi, kp, p.k_sb, p.k_sh, p.k_st, Ks, Dp);
      load_key_tile<T>(p, g, b, kvh, kb, k_hi, vp, p.v_sb, p.v_sh, p.v_st, Vs, Dp);
      __syncthreads();
      float z = score(kb);
      float m_new = fmaxf(m, warp_max(z));
      float alpha = exp2f(m - m_new);
      float pj = (z == kNegInf) ? 0.f : exp2f(z - m_new);
      l = l * alpha + warp_sum(pj);
#pragma unroll
      for (int i = 0; i < kMaxDimRegs; ++i) acc[i] *= alpha;
      accumulate_pv(pj);
      m = m_new;
    }
    float inv = 1.f / l;
#pragma unroll
    for (int i = 0; i < kMaxDimRegs; ++i) acc[i] *= inv;
    stat0 = m;
    stat1 = l;
  } else {
    // Pass 1: row max.
    float zmax = kNegInf;
    for (int kb = k_lo; kb < k_hi; kb += kTile) {
      __syncthreads();
      load_key_tile<T>(p, g, b, kvh, kb, k_hi, kp, p.k_sb, p.k_sh, p.k_st, Ks, Dp);
      __syncthreads();
      zmax = fmaxf(zmax, warp_max(score(kb)));
    }
    const bool empty = !(zmax > kNegInf);
    bool done = empty || !active;
    float t = zmax - 1.f, tau = kPosInf;
    // Exact threshold: bracket sweeps until the candidate set is the support.
    for (int it = 0; it < 64; ++it) {
      if (!__syncthreads_or(!done)) break;
      TauStats st{0.f, 0.f, 0.f, kPosInf};
      for (int kb = k_lo; kb < k_hi; kb += kTile) {
        __syncthreads();
        load_key_tile<T>(p, g, b, kvh, kb, k_hi, kp, p.k_sb, p.k_sh, p.k_st, Ks, Dp);
        __syncthreads();
        float z = score(kb);
        if (!done) tau_accumulate(st, z, t);
      }
      st.cnt = warp_sum(st.cnt);
      st.s1 = warp_sum(st.s1);
      st.s2 = warp_sum(st.s2);
      st.zmin = warp_min(st.zmin);
      if (!done) done = tau_step(NORM, st, &t, &tau);
    }
    float support = 0.f;
    for (int kb = k_lo; kb < k_hi; kb += kTile) {
      __syncthreads();
      load_key_tile<T>(p, g, b, kvh, kb, k_hi, kp, p.k_sb, p.k_sh, p.k_st, Ks, Dp);
      load_key_tile<T>(p, g, b, kvh, kb, k_hi, vp, p.v_sb, p.v_sh, p.v_st, Vs, Dp);
      __syncthreads();
      float z = score(kb);
      float pj = (active && !empty) ? sparse_prob(NORM, z, tau) : 0.f;
      support += warp_sum(pj > 0.f ? 1.f : 0.f);
      accumulate_pv(pj);
    }
    stat0 = empty ? kPosInf : tau;
    stat1 = support;
  }

  if (active) {
    T* op = static_cast<T*>(p.o) + qrow_off(p, g, b, h, row, p.o_sb, p.o_sh, p.o_st);
#pragma unroll
    for (int i = 0; i < kMaxDimRegs; ++i) {
      int d = lane + 32 * i;
      if (d < D) op[d] = from_f32<T>(acc[i]);
    }
    if (lane == 0) {
      int64_t si = stat_index(p, g, h, row);
      p.stats[si] = stat0;
      p.stats[(int64_t)p.hq * p.rows_total + si] = stat1;
    }
  }
}

// --------------------------------------------------------------------------
// Backward, query side: per-row correction term and dQ.
// --------------------------------------------------------------------------
template <typename T, typename G, int NORM>
__global__ void __launch_bounds__(kRows * 32) simt_bwd_dq_kernel(AttnParams p) {
  extern __shared__ float smem[];
  const int D = p.d, Dp = D + 1;
  float* Ks = smem;
  float* Vs = Ks + kTile * Dp;
  float* Qs = Vs + kTile * Dp;   // [8][D]
  float* dOs = Qs + kRows * D;   // [8][D]
  const int b = blockIdx.z, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Geometry g = geometry(p, b);
  const int q0 = blockIdx.x * kRows;
  if (q0 >= g.q_len) return;
  const int row = q0 + warp;
  const bool active = row < g.q_len;
  const int kvh = h / (p.hq / p.hkv);
  const T* kp = static_cast<const T*>(p.k);
  const T* vp = static_cast<const T*>(p.v);

  float corr_part = 0.f;
  {
    const T* qp = static_cast<const T*>(p.q);
    const T* dop = static_cast<const T*>(p.dout);
    const T* opp = static_cast<const T*>(p.o);
    int64_t qo = qrow_off(p, g, b, h, row, p.q_sb, p.q_sh, p.q_st);
    int64_t doo = qrow_off(p, g, b, h, row, p.do_sb, p.do_sh, p.do_st);
    int64_t oo = qrow_off(p, g, b, h, row, p.o_sb, p.o_sh, p.o_st);
    for (int d = lane; d < D; d += 32) {
      float dov = active ? to_f32<T>(dop[doo + d]) : 0.f;
      Qs[warp * D + d] = active ? to_f32<T>(qp[qo + d]) : 0.f;
      dOs[warp * D + d] = dov;
      if (NORM == HFAN_SOFTMAX1 && active) corr_part += dov * to_f32<T>(opp[oo + d]);
    }
  }
  float st0 = 0.f, st1 = 1.f;
  if (active) {
    int64_t si = stat_index(p, g, h, row);
    st0 = p.stats[si];
    st1 = p.stats[(int64_t)p.hq * p.rows_total + si];
  }
  const bool empty = (NORM != HFAN_SOFTMAX1) && !(st0 < kPosInf);

  const int last_row = min(q0 + kRows - 1, g.q_len - 1);
  int k_hi = g.k_len;
  if (p.causal) k_hi = min(k_hi, last_row + g.shift + 1);
  int k_lo = 0;
  if (p.window_left > 0) k_lo = max(0, q0 + g.shift - p.window_left + 1);
  k_lo = (k_lo / kTile) * kTile;
  const float zs = zscale_of<NORM>(p.scale);
  const float inv_l = 1.f / st1;

  auto load_kv = [&](int kb) {
    __syncthreads();
    load_key_tile<T>(p, g, b, kvh, kb, k_hi, kp, p.k_sb, p.k_sh, p.k_st, Ks, Dp);
    load_key_tile<T>(p, g, b, kvh, kb, k_hi, vp, p.v_sb, p.v_sh, p.v_st, Vs, Dp);
    __syncthreads();
  };
  // Per-key probability p and inverse-Hessian weight w for this lane's key.
  auto prob = [&](int kb, float* w) -> float {
    int j = kb + lane;
    bool vis = active && !empty && key_visible(row, j, g, p.causal, p.window_left);
    float z = dot_row(Qs + warp * D, Ks + lane * Dp, D) * zs;
    if (!vis) {
      *w = 0.f;
      return 0.f;
    }
    if (NORM == HFAN_SOFTMAX1) {
      float pj = exp2f(z - st0) * inv_l;
      *w = pj;
      return pj;
    }
    *w = sparse_g(NORM, z, st0);
    return sparse_prob(NORM, z, st0);
  };

  float c;
  if (NORM == HFAN_SOFTMAX1) {
    // sum_j p_j dP_j = dO . O because the implicit sink has value 0.
    c = warp_sum(corr_part);
  } else {
    float num = 0.f, den = 0.f;
    for (int kb = k_lo; kb < k_hi; kb += kTile) {
      load_kv(kb);
      float w;
      prob(kb, &w);
      if (w != 0.f) {
        float dp = dot_row(dOs + warp * D, Vs + lane * Dp, D);
        num = fmaf(w, dp, num);
        den += w;
      }
    }
    num = warp_sum(num);
    den = warp_sum(den);
    c = den > 0.f ? num / den : 0.f;
  }
  if (active && lane == 0) p.corr[stat_index(p, g, h, row)] = c;

  float acc[kMaxDimRegs];
#pragma unroll
  for (int i = 0; i < kMaxDimRegs; ++i) acc[i] = 0.f;
  for (int kb = k_lo; kb < k_hi; kb += kTile) {
    load_kv(kb);
    float w;
    prob(kb, &w);
    float ds = 0.f;
    if (w != 0.f) {
      float dp = dot_row(dOs + warp * D, Vs + lane * Dp, D);
      ds = w * (dp - c);
    }
    for (int jj = 0; jj < kTile; ++jj) {
      float dr = __shfl_sync(0xffffffffu, ds, jj);
      if (dr != 0.f) {
#pragma unroll
        for (int i = 0; i < kMaxDimRegs; ++i) {
          int d = lane + 32 * i;
          if (d < D) acc[i] = fmaf(dr, Ks[jj * Dp + d], acc[i]);
        }
      }
    }
  }
  if (active) {
    G* dqp = static_cast<G*>(p.dq) + qrow_off(p, g, b, h, row, p.dq_sb, p.dq_sh, p.dq_st);
#pragma unroll
    for (int i = 0; i < kMaxDimRegs; ++i) {
      int d = lane + 32 * i;
      if (d < D) dqp[d] = from_f32<G>(acc[i] * p.scale);
    }
  }
}

// --------------------------------------------------------------------------
// Backward, key side: dK and dV, one warp per key.
// --------------------------------------------------------------------------
template <typename T, typename G, int NORM>
__global__ void __launch_bounds__(kRows * 32) simt_bwd_dkdv_kernel(AttnParams p) {
  extern __shared__ float smem[];
  const int D = p.d, Dp = D + 1;
  float* Qt = smem;               // [32][Dp]
  float* dOt = Qt + kTile * Dp;   // [32][Dp]
  float* Kw = dOt + kTile * Dp;   // [8][D]
  float* Vw = Kw + kRows * D;     // [8][D]
  float* rs0 = Vw + kRows * D;    // [32] stats0
  float* rs1 = rs0 + kTile;       // [32] stats1
  float* rc = rs1 + kTile;        // [32] corr
  const int b = blockIdx.z, kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Geometry g = geometry(p, b);
  const int k0 = blockIdx.x * kRows;
  if (k0 >= g.k_len) return;
  const int j = k0 + warp;
  const bool active = j < g.k_len;
  const int groups = p.hq / p.hkv;
  const T* qp = static_cast<const T*>(p.q);
  const T* dop = static_cast<const T*>(p.dout);

  int64_t ktok = -1;
  if (active) ktok = key_token(p, g, b, j);
  {
    const T* kp = static_cast<const T*>(p.k);
    const T* vp = static_cast<const T*>(p.v);
    for (int d = lane; d < D; d += 32) {
      bool ok = ktok >= 0;
      Kw[warp * D + d] = ok ? to_f32<T>(kp[key_off(p, b, kvh, ktok, p.k_sb, p.k_sh, p.k_st) + d]) : 0.f;
      Vw[warp * D + d] = ok ? to_f32<T>(vp[key_off(p, b, kvh, ktok, p.v_sb, p.v_sh, p.v_st) + d]) : 0.f;
    }
  }
  // Query rows that can see any key of this CTA.
  const int off = g.shift;  // key j visible to row i iff j <= i + off (causal)
  int i_lo = 0;
  if (p.causal) i_lo = max(0, k0 - off);
  int i_hi = g.q_len;
  if (p.window_left > 0) i_hi = min(i_hi, k0 + kRows - 1 - off + p.window_left);
  i_lo = (i_lo / kTile) * kTile;
  const float zs = zscale_of<NORM>(p.scale);

  float dk[kMaxDimRegs], dv[kMaxDimRegs];
#pragma unroll
  for (int i = 0; i < kMaxDimRegs; ++i) dk[i] = dv[i] = 0.f;

  for (int gi = 0; gi < groups; ++gi) {
    const int h = kvh * groups + gi;
    for (int i0 = i_lo; i0 < i_hi; i0 += kTile) {
      __syncthreads();
      for (int idx = threadIdx.x; idx < kTile * D; idx += blockDim.x) {
        int r = idx / D, c = idx - r * D;
        int i = i0 + r;
        float qv = 0.f, dov = 0.f;
        if (i < g.q_len) {
          qv = to_f32<T>(qp[qrow_off(p, g, b, h, i, p.q_sb, p.q_sh, p.q_st) + c]);
          dov = to_f32<T>(dop[qrow_off(p, g, b, h, i, p.do_sb, p.do_sh, p.do_st) + c]);
        }
        Qt[r * Dp + c] = qv;
        dOt[r * Dp + c] = dov;
      }
      if (threadIdx.x < kTile) {
        int i = i0 + threadIdx.x;
        float a = 0.f, bb = 1.f, cc = 0.f;
        if (i < g.q_len) {
          int64_t si = stat_index(p, g, h, i);
          a = p.stats[si];
          bb = p.stats[(int64_t)p.hq * p.rows_total + si];
          cc = p.corr[si];
        }
        rs0[threadIdx.x] = a;
        rs1[threadIdx.x] = bb;
        rc[threadIdx.x] = cc;
      }
      __syncthreads();
      const int i = i0 + lane;
      bool vis = active && ktok >= 0 && i < g.q_len && key_visible(i, j, g, p.causal, p.window_left);
      float pj = 0.f, ds = 0.f;
      if (vis) {
        float z = dot_row(Qt + lane * Dp, Kw + warp * D, D) * zs;
        float dp = dot_row(dOt + lane * Dp, Vw + warp * D, D);
        float w;
        if (NORM == HFAN_SOFTMAX1) {
          pj = exp2f(z - rs0[lane]) / rs1[lane];
          w = pj;
        } else {
          pj = sparse_prob(NORM, z, rs0[lane]);
          w = sparse_g(NORM, z, rs0[lane]);
        }
        ds = w * (dp - rc[lane]);
      }
      for (int rr = 0; rr < kTile; ++rr) {
        float pr = __shfl_sync(0xffffffffu, pj, rr);
        float dr = __shfl_sync(0xffffffffu, ds, rr);
        if (pr != 0.f || dr != 0.f) {
#pragma unroll
          for (int k = 0; k < kMaxDimRegs; ++k) {
            int d = lane + 32 * k;
            if (d < D) {
              dv[k] = fmaf(pr, dOt[rr * Dp + d], dv[k]);
              dk[k] = fmaf(dr, Qt[rr * Dp + d], dk[k]);
            }
          }
        }
      }
    }
  }
  if (active && ktok >= 0) {
    if (p.paged) {
      float* dkp = static_cast<float*>(p.dk) + key_off(p, b, kvh, ktok, p.dk_sb, p.dk_sh, p.dk_st);
      float* dvp = static_cast<float*>(p.dv) + key_off(p, b, kvh, ktok, p.dv_sb, p.dv_sh, p.dv_st);
#pragma unroll
      for (int k = 0; k < kMaxDimRegs; ++k) {
        int d = lane + 32 * k;
        if (d < D) {
          atomicAdd(dkp + d, dk[k] * p.scale);
          atomicAdd(dvp + d, dv[k]);
        }
      }
    } else {
      G* dkp = static_cast<G*>(p.dk) + key_off(p, b, kvh, ktok, p.dk_sb, p.dk_sh, p.dk_st);
      G* dvp = static_cast<G*>(p.dv) + key_off(p, b, kvh, ktok, p.dv_sb, p.dv_sh, p.dv_st);
#pragma unroll
      for (int k = 0; k < kMaxDimRegs; ++k) {
        int d = lane + 32 * k;
        if (d < D) {
          dkp[d] = from_f32<G>(dk[k] * p.scale);
          dvp[d] = from_f32<G>(dv[k]);
        }
      }
    }
  }
}

// --------------------------------------------------------------------------
// Launchers
// --------------------------------------------------------------------------
size_t simt_fwd_smem(int D) { return sizeof(float) * (2 * kTile * (D + 1) + kRows * D); }
size_t simt_dq_smem(int D) { return sizeof(float) * (2 * kTile * (D + 1) + 2 * kRows * D); }
size_t simt_dkdv_smem(int D) {
  return sizeof(float) * (2 * kTile * (D + 1) + 2 * kRows * D + 3 * kTile);
}

template <typename K>
static cudaError_t launch(K kernel, dim3 grid, size_t smem, cudaStream_t stream, const AttnParams& p) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kernel<<<grid, kRows * 32, smem, stream>>>(p);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t fwd_t(const AttnParams& p, int max_q, cudaStream_t s) {
  dim3 grid((max_q + kRows - 1) / kRows, p.hq, p.batch);
  size_t sm = simt_fwd_smem(p.d);
  switch (p.norm) {
    case HFAN_SOFTMAX1: return launch(simt_fwd_kernel<T, HFAN_SOFTMAX1>, grid, sm, s, p);
    case HFAN_SPARSEMAX: return launch(simt_fwd_kernel<T, HFAN_SPARSEMAX>, grid, sm, s, p);
    default: return launch(simt_fwd_kernel<T, HFAN_ENTMAX15>, grid, sm, s, p);
  }
}

template <typename T, typename G>
static cudaError_t bwd_tg(const AttnParams& p, int max_q, int max_k, cudaStream_t s) {
  dim3 gq((max_q + kRows - 1) / kRows, p.hq, p.batch);
  dim3 gk((max_k + kRows - 1) / kRows, p.hkv, p.batch);
  cudaError_t e;
  switch (p.norm) {
    case HFAN_SOFTMAX1:
      e = launch(simt_bwd_dq_kernel<T, G, HFAN_SOFTMAX1>, gq, simt_dq_smem(p.d), s, p);
      if (e != cudaSuccess) return e;
      return launch(simt_bwd_dkdv_kernel<T, G, HFAN_SOFTMAX1>, gk, simt_dkdv_smem(p.d), s, p);
    case HFAN_SPARSEMAX:
      e = launch(simt_bwd_dq_kernel<T, G, HFAN_SPARSEMAX>, gq, simt_dq_smem(p.d), s, p);
      if (e != cudaSuccess) return e;
      return launch(simt_bwd_dkdv_kernel<T, G, HFAN_SPARSEMAX>, gk, simt_dkdv_smem(p.d), s, p);
    default:
      e = launch(simt_bwd_dq_kernel<T, G, HFAN_ENTMAX15>, gq, simt_dq_smem(p.d), s, p);
      if (e != cudaSuccess) return e;
      return launch(simt_bwd_dkdv_kernel<T, G, HFAN_ENTMAX15>, gk, simt_dkdv_smem(p.d), s, p);
  }
}

cudaError_t simt_attention_fwd(int dtype, const AttnParams& p, int max_q, cudaStream_t s) {
  switch (dtype) {
    case HFAN_FLOAT32: return fwd_t<float>(p, max_q, s);
    case HFAN_FLOAT16: return fwd_t<__half>(p, max_q, s);
    default: return fwd_t<__nv_bfloat16>(p, max_q, s);
  }
}

// Gradients are written in float32 when p.grad_f32 (always for the paged
// layout, whose shared pages accumulate atomically), else in the input type.
cudaError_t simt_attention_bwd(int dtype, const AttnParams& p, int max_q, int max_k, cudaStream_t s) {
  if (p.grad_f32 || p.paged) {
    switch (dtype) {
      case HFAN_FLOAT32: return bwd_tg<float, float>(p, max_q, max_k, s);
      case HFAN_FLOAT16: return bwd_tg<__half, float>(p, max_q, max_k, s);
      default: return bwd_tg<__nv_bfloat16, float>(p, max_q, max_k, s);
    }
  }
  switch (dtype) {
    case HFAN_FLOAT32: return bwd_tg<float, float>(p, max_q, max_k, s);
    case HFAN_FLOAT16: return bwd_tg<__half, __half>(p, max_q, max_k, s);
    default: return bwd_tg<__nv_bfloat16, __nv_bfloat16>(p, max_q, max_k, s);
  }
}

}  // namespace hfan
