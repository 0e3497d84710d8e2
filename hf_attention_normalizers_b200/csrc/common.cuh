// Shared device helpers: element conversion, warp reductions, the exact
// threshold (tau) solver used by sparsemax / entmax15, and the kernel-side
// parameter blocks.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hfan.h"

namespace hfan {

constexpr float kNegInf = -__builtin_huge_valf();
constexpr float kPosInf = __builtin_huge_valf();
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// element <-> float
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Exact threshold solve.
//
// Both sparse normalizers are p_i = (z_i - tau)_+^a with sum_i p_i = 1, a = 1
// (sparsemax, z = s) or a = 2 (entmax15, z = s / 2).  The reference finds tau by
// sorting each row (vutils/entmax.py:35-133).  Here tau is found from a
// bracket and the closed form on the support:
//
//   * any row has tau >= zmax - 1, because the top entry alone has
//     (zmax - tau)^a <= 1; so keys with z <= zmax - 1 are never in the support.
//   * given a lower bound t <= tau, one sweep over the row gathers, over the
//     candidate set S = {z > t}: cnt = |S|, s1 = sum (z - t), s2 = sum (z - t)^2
//     and zmin = min_S z.  The closed-form threshold of S is
//         sparsemax:  tc = t + (s1 - 1) / cnt
//         entmax15:   tc = t + (s1 - sqrt(s1^2 - cnt (s2 - 1))) / cnt
//     (the entmax root is the vutils formula mean - sqrt((1 - ss)/rho) written
//     around t).  If zmin >= tc the candidate set is exactly the support and
//     tc is the exact threshold.  Otherwise the row is refined with a Newton
//     step on f(t) = sum (z - t)_+^a - 1 (convex and decreasing, so Newton from
//     the left never overshoots): sparsemax t <- tc (Michelot's iteration),
//     entmax15 t <- t + (s2 - 1) / (2 s1).
//
// The sums may be taken relative to any fixed reference r instead of t
// (s1 = sum (z - r), s2 = sum (z - r)^2 over the same set S = {z > t}); the
// closed form is then evaluated around r.  With r = the row maximum the result
// depends only on the set S and the order of summation, not on the lower
// bound t that found S; the tensor-core forward uses that to make tau
// bit-reproducible, and it is the reference's own form (vutils works on
// X - max).
// ---------------------------------------------------------------------------
struct TauStats {
  float cnt, s1, s2, zmin;
};

__device__ __forceinline__ void tau_accumulate_ref(TauStats& st, float z, float t, float r) {
  if (z > t) {
    float d = z - r;
    st.cnt += 1.f;
    st.s1 += d;
    st.s2 += d * d;
    st.zmin = fminf(st.zmin, z);
  }
}

__device__ __forceinline__ void tau_accumulate(TauStats& st, float z, float t) { tau_accumulate_ref(st, z, t, t); }

// Sums taken around r.  Returns true when t is resolved and writes the exact
// threshold to *tau.  On false, *t holds the refined lower bound for the next
// sweep and *tau the current closed-form estimate.
__device__ __forceinline__ bool tau_step_ref(int norm, const TauStats& st, float r, float* t, float* tau) {
  const float cnt = fmaxf(st.cnt, 1.f);
  float tc;
  if (norm == HFAN_SPARSEMAX) {
    tc = r + (st.s1 - 1.f) / cnt;
  } else {
    const float disc = fmaxf(st.s1 * st.s1 - cnt * (st.s2 - 1.f), 0.f);
    tc = r + (st.s1 - sqrtf(disc)) / cnt;
  }
  *tau = tc;
  if (st.zmin >= tc) return true;
  float nt;
  if (norm == HFAN_SPARSEMAX) {
    nt = tc;
  } else {
    // Newton step on sum (z - t)^2 - 1: the sums around t from those around r
    const float dl = r - *t;
    const float s1t = st.s1 + st.cnt * dl;
    const float s2t = st.s2 + dl * (2.f * st.s1 + st.cnt * dl);
    nt = *t + (s2t - 1.f) / (2.f * fmaxf(s1t, 1e-30f));
  }
  // Guard against a rounding stall: the next bound must strictly grow.
  *t = fmaxf(nt, nextafterf(*t, kPosInf));
  return false;
}

// Sums taken around t itself.
__device__ __forceinline__ bool tau_step(int norm, const TauStats& st, float* t, float* tau) {
  return tau_step_ref(norm, st, *t, t, tau);
}

__device__ __forceinline__ float sparse_prob(int norm, float z, float tau) {
  float d = fmaxf(z - tau, 0.f);
  return norm == HFAN_SPARSEMAX ? d : d * d;
}
// g = 1[p>0] (sparsemax) or sqrt(p) (entmax15): the diagonal of the inverse
// Hessian used by both closed-form backwards (vutils/entmax.py:148-157, 175-183).
__device__ __forceinline__ float sparse_g(int norm, float z, float tau) {
  float d = z - tau;
  if (!(d > 0.f)) return 0.f;
  return norm == HFAN_SPARSEMAX ? 1.f : d;
}

// ---------------------------------------------------------------------------
// Sequence geometry shared by the attention kernels.
// ---------------------------------------------------------------------------
struct Geometry {
  int q_start, q_len;   // first packed row / number of query rows of this sequence
  int k_start, k_len;   // first packed key / number of keys
  int shift;            // causal alignment: row i sees keys j <= i + shift (k_len - q_len,
                        // bottom-right; 0 with causal_top_left)
};

__device__ __forceinline__ bool key_visible(int i, int j, const Geometry& g, int causal,
                                            int window_left) {
  if (j >= g.k_len) return false;
  int limit = i + g.shift;
  if (causal && j > limit) return false;
  if (window_left > 0 && j <= limit - window_left) return false;
  return true;
}

// Device-side status word: kernels record the first error they detect
// (out-of-range page id, bounded wait expired) instead of trapping.
enum DeviceError : int {
  kDevOk = 0,
  kDevBadPage = 1,
  kDevWaitTimeout = 2,
  kDevBadLength = 3,
};

}  // namespace hfan

namespace hfan {

// ---------------------------------------------------------------------------
// Dropout mask: a counter-based generator, so that the forward and both
// backward kernels regenerate the same keep bits from the saved seed instead
// of storing a [B, H, Lq, Lk] mask (the reference does the same with Triton's
// tl.rand, kernels/softmax1_hopper.py:105-110, sparse_entmax_hopper.py:141-145).
//
// Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC 2011): ten rounds of two 32x32->64-bit products with the
// multipliers 0xD2511F53 / 0xCD9E8D57, the key bumped by the Weyl constants
// 0x9E3779B9 / 0xBB67AE85 between rounds.
//
// Element (row r, key j), r = (b * heads_q + h) * len_q + i: counter
// (j / 4, r lo, r hi, 0), key (seed lo, seed hi), word j % 4; its top 24 bits
// u give keep = u >= ceil(p 2^24) (i.e. uniform >= p).  Four consecutive keys
// of a row share one generator call.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// Keep bits (bit e = key 4 g + e) of one group of four keys of row r.
__device__ __forceinline__ uint32_t dropout_keep4(uint64_t r, uint32_t g, uint32_t seed_lo, uint32_t seed_hi,
                                                  uint32_t thr24) {
  const uint4 x = philox4x32_10(make_uint4(g, (uint32_t)r, (uint32_t)(r >> 32), 0u), seed_lo, seed_hi);
  return ((x.x >> 8) >= thr24 ? 1u : 0u) | ((x.y >> 8) >= thr24 ? 2u : 0u) | ((x.z >> 8) >= thr24 ? 4u : 0u) |
         ((x.w >> 8) >= thr24 ? 8u : 0u);
}

}  // namespace hfan
