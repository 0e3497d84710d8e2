// Sparse backward of the sparse normalizers from the forward's support lists.
//
// The tile kernels (tc_backward.cu) recompute S and dP for every 128 x 128
// tile and apply dS = w (dP - c) to all of it, although w is zero outside the
// support: on random scores sparsemax keeps about 5 keys of a 4096-key row
// and entmax15 about 25.  When the forward wrote every row's support list
// (keys with p > 0, see AttnParams::sl_key), dQ only needs those keys:
//
//   dP_j = dO . v_j                        for j in the support
//   c    = sum_j w_j dP_j / sum_j w_j      (w = 1 for sparsemax, sqrt(p) for entmax15)
//   dS_j = w_j (dP_j - c),   dQ = scale sum_j dS_j k_j
//
// the closed-form backwards of vutils/entmax.py:148-157 and :175-183 that the
// tile kernels apply.  Four lanes (a quad) share a row, each owning a quarter
// of the head dimension; dot products are reduced across the quad with
// shuffles.  Summation follows the list order (sub-list by sub-list, keys in
// increasing order), so results are the same on every run.  c goes to the
// corr buffer for the dK/dV kernel and dS_j to sl_g.  When some list
// overflowed (sl_flag != 0) the kernel returns at once and the tile kernels
// run instead.
#include "common.cuh"
#include "params.cuh"

namespace hfan {
namespace {

template <bool BF16>
__device__ __forceinline__ void unpack8(const uint4& x, float (&f)[8]) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (BF16) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    } else {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if (BF16) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

constexpr int kRowsPerBlock = 64;  // 256 threads: 64 rows x 4 lanes

template <int HD, bool BF16, int NORM>
__global__ void __launch_bounds__(256) sparse_dq_kernel(const AttnParams p) {
  if (*p.sl_flag != 0) return;  // a list overflowed: the tile kernels run
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int NWG = HD / 32;          // sub-lists per row
  constexpr int LW = kSupSlots / NWG;   // slots per sub-list
  constexpr int DL = HD / 4;            // head-dim columns per lane
  constexpr int NV = DL / 8;            // 16-byte vectors per lane and row
  const int lane = threadIdx.x & 31;
  const int q = lane & 3;
  const unsigned qmask = 0xfu << (lane & ~3);
  const int h = blockIdx.y;
  const int r = blockIdx.x * kRowsPerBlock + (threadIdx.x >> 2);
  if (r >= p.rows_total) return;  // whole quads leave together
  const int kvh = h / (p.hq / p.hkv);
  // stats row -> (sequence, token): dense rows are b * len_q + i; packed
  // varlen rows are tokens (no batch stride)
  const bool varlen = p.cu_q != nullptr;
  const int b = varlen ? 0 : r / p.len_q;
  const int64_t tq = varlen ? r : r % p.len_q;
  const int64_t kbase_b = varlen ? 0 : (int64_t)b;

  float dof[DL];
  {
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const T*>(p.dout) + (int64_t)b * p.do_sb +
                                                      (int64_t)h * p.do_sh + tq * p.do_st + q * DL);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float f[8];
      unpack8<BF16>(src[v], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) dof[v * 8 + e] = f[e];
    }
  }
  const T* vb = static_cast<const T*>(p.v) + kbase_b * p.v_sb + (int64_t)kvh * p.v_sh + q * DL;
  const T* kb = static_cast<const T*>(p.k) + kbase_b * p.k_sb + (int64_t)kvh * p.k_sh + q * DL;

  int cnt[NWG];
#pragma unroll
  for (int w = 0; w < NWG; ++w) cnt[w] = p.sl_cnt[((int64_t)h * p.rows_total + r) * NWG + w];
  const int64_t row_slots = ((int64_t)h * p.rows_total + r) * kSupSlots;

  // pass 1: dP_j and the correction sums
  float num = 0.f, den = 0.f;
#pragma unroll
  for (int w = 0; w < NWG; ++w) {
    for (int e = 0; e < cnt[w]; ++e) {
      const int64_t slot = row_slots + w * LW + e;
      const int2 ent = p.sl_ent[slot];
      const int key = ent.x;
      const float pv = __int_as_float(ent.y);
      const uint4* src = reinterpret_cast<const uint4*>(vb + (int64_t)key * p.v_st);
      float part = 0.f;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float f[8];
        unpack8<BF16>(__ldg(src + v), f);
#pragma unroll
        for (int x = 0; x < 8; ++x) part = fmaf(dof[v * 8 + x], f[x], part);
      }
      part += __shfl_xor_sync(qmask, part, 1);
      part += __shfl_xor_sync(qmask, part, 2);
      const float wt = NORM == HFAN_SPARSEMAX ? 1.f : sqrtf(pv);
      num = fmaf(wt, part, num);
      den += wt;
      if (q == 0) p.sl_g[slot] = part;
    }
  }
  const float c = den > 0.f ? num / den : 0.f;
  __syncwarp(qmask);  // lane 0's dP values are visible to the quad

  // pass 2: dS_j and dQ
  float acc[DL];
#pragma unroll
  for (int x = 0; x < DL; ++x) acc[x] = 0.f;
#pragma unroll
  for (int w = 0; w < NWG; ++w) {
    for (int e = 0; e < cnt[w]; ++e) {
      const int64_t slot = row_slots + w * LW + e;
      const int2 ent = p.sl_ent[slot];
      const int key = ent.x;
      const float pv = __int_as_float(ent.y);
      const float dp = p.sl_g[slot];
      const float wt = NORM == HFAN_SPARSEMAX ? 1.f : sqrtf(pv);
      const float ds = wt * (dp - c);
      const uint4* src = reinterpret_cast<const uint4*>(kb + (int64_t)key * p.k_st);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        float f[8];
        unpack8<BF16>(__ldg(src + v), f);
#pragma unroll
        for (int x = 0; x < 8; ++x) acc[v * 8 + x] = fmaf(ds, f[x], acc[v * 8 + x]);
      }
      __syncwarp(qmask);  // every lane has read dP before lane 0 replaces it
      if (q == 0) p.sl_g[slot] = ds;
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(p.dq) + (int64_t)b * p.dq_sb + (int64_t)h * p.dq_sh +
                                        tq * p.dq_st + q * DL);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    uint4 o;
    o.x = pack_pair<BF16>(acc[v * 8 + 0] * p.scale, acc[v * 8 + 1] * p.scale);
    o.y = pack_pair<BF16>(acc[v * 8 + 2] * p.scale, acc[v * 8 + 3] * p.scale);
    o.z = pack_pair<BF16>(acc[v * 8 + 4] * p.scale, acc[v * 8 + 5] * p.scale);
    o.w = pack_pair<BF16>(acc[v * 8 + 6] * p.scale, acc[v * 8 + 7] * p.scale);
    dst[v] = o;
  }
  if (q == 0) p.corr[(int64_t)h * p.rows_total + r] = c;
}

template <int HD, bool BF16>
cudaError_t launch_dq(const AttnParams& p, cudaStream_t s) {
  const dim3 grid((p.rows_total + kRowsPerBlock - 1) / kRowsPerBlock, p.hq);
  if (p.norm == HFAN_SPARSEMAX)
    sparse_dq_kernel<HD, BF16, HFAN_SPARSEMAX><<<grid, 256, 0, s>>>(p);
  else
    sparse_dq_kernel<HD, BF16, HFAN_ENTMAX15><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

// dQ and the row correction from the support lists (no-op on the device when
// a list overflowed).  16-bit inputs and gradients, head_dim 64 or 128.
cudaError_t sparse_list_dq(int dtype, const AttnParams& p, cudaStream_t s) {
  const bool bf16 = dtype == HFAN_BFLOAT16;
  if (p.d == 128) return bf16 ? launch_dq<128, true>(p, s) : launch_dq<128, false>(p, s);
  return bf16 ? launch_dq<64, true>(p, s) : launch_dq<64, false>(p, s);
}

}  // namespace hfan
