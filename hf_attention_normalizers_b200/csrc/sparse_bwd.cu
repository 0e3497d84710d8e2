// Sparse backward of the sparse normalizers from the forward's support lists.
//
// The tile kernels (tc_backward.cu) recompute S and dP for every 128 x 128
// tile and apply dS = w (dP - c) to all of it, although w is zero outside the
// support: on random scores sparsemax keeps about 5 keys of a 4096-key row
// and entmax15 about 25.  When the forward wrote every row's support list
// (keys with p > 0, see AttnParams::sl_ent), dQ only needs those keys:
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

#include <climits>

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
  if (*p.sl_flag & kListRowOverflow) return;  // a row list overflowed: the tile kernels run
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
      if (q == 0) {
        p.sl_g[slot] = ds;
        atomicAdd(p.sl_kcnt + list_kid(p, b, kvh, key), 1);  // the key side's entry count
      }
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

// ---- key side: dK_j = scale sum_i dS_ij q_i and dV_j = sum_i p_ij dO_i over
// the rows i whose lists hold key j.  The entries are counted per key by the
// dQ kernel, offset by a two-kernel prefix over the key counters, scattered
// into key order by key_fill_kernel and sorted by slot number within each key
// (slot order is (query head, row) order), so every dK/dV sum runs in the
// same order on every run.

// Sum of each kKeyScanBlock block of key counters.
__global__ void __launch_bounds__(256) key_block_sum_kernel(const AttnParams p) {
  if (*p.sl_flag != 0) return;
  __shared__ int part[8];
  const int64_t base = (int64_t)blockIdx.x * kKeyScanBlock;
  int sum = 0;
  for (int i = threadIdx.x; i < kKeyScanBlock; i += 256) {
    const int64_t k = base + i;
    sum += k < p.sl_nk ? p.sl_kcnt[k] : 0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < 8; ++w) t += part[w];
    p.sl_bsum[blockIdx.x] = t;
    if (blockIdx.x == 0) p.sl_long[0] = 0;  // no long key yet (key_scan_kernel runs next)
  }
}

// Exclusive prefix of the key counters into sl_koff (and the fill cursors in
// sl_kcnt); keys with more than kKeyMaxEntries entries go to the long-key list.
__global__ void __launch_bounds__(256) key_scan_kernel(const AttnParams p) {
  if (*p.sl_flag != 0) return;
  constexpr int PER = kKeyScanBlock / 256;  // consecutive counters per thread
  __shared__ int wsum[8];
  __shared__ int carry;
  if (threadIdx.x < 32) {  // the sums of all earlier blocks
    int c = 0;
    for (int j = threadIdx.x; j < (int)blockIdx.x; j += 32) c += p.sl_bsum[j];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if (threadIdx.x == 0) carry = c;
  }
  const int64_t base = (int64_t)blockIdx.x * kKeyScanBlock + threadIdx.x * PER;
  int v[PER];
  int tsum = 0;
  bool longk = false;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    v[e] = base + e < p.sl_nk ? p.sl_kcnt[base + e] : 0;
    longk |= v[e] > kKeyMaxEntries;
    tsum += v[e];
  }
  if (longk) {
    for (int e = 0; e < PER; ++e) {
      if (v[e] <= kKeyMaxEntries) continue;
      const int i = atomicAdd(p.sl_long, 1);
      if (i < p.sl_long_cap)
        p.sl_long[1 + i] = (int)(base + e);
      else
        atomicOr(p.sl_flag, kListKeyOverflow);
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = tsum;  // inclusive warp scan of the thread sums
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  int off = carry + incl - tsum;
  for (int w = 0; w < warp; ++w) off += wsum[w];
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    if (base + e < p.sl_nk) {
      p.sl_koff[base + e] = off;
      p.sl_kcnt[base + e] = off;
    }
    off += v[e];
  }
  if (base + PER >= p.sl_nk && base < p.sl_nk) p.sl_koff[p.sl_nk] = off;  // the thread holding the last key
}

// Scatter the slot numbers of every sub-list into their keys' segments.
template <int HD>
__global__ void __launch_bounds__(256) key_fill_kernel(const AttnParams p) {
  if (*p.sl_flag != 0) return;
  constexpr int NWG = HD / 32;
  constexpr int LW = kSupSlots / NWG;
  const int64_t idx = (int64_t)blockIdx.x * 256 + threadIdx.x;  // (h, r, w)
  if (idx >= (int64_t)p.hq * p.rows_total * NWG) return;
  const int w = (int)(idx % NWG);
  const int64_t hr = idx / NWG;
  const int h = (int)(hr / p.rows_total);
  const int r = (int)(hr - (int64_t)h * p.rows_total);
  const int kvh = h / (p.hq / p.hkv);
  const int b = p.cu_q != nullptr ? 0 : r / p.len_q;
  const int n = p.sl_cnt[idx];
  const int slot0 = (int)(hr * kSupSlots + w * LW);
  for (int e = 0; e < n; ++e) {
    const int key = p.sl_ent[slot0 + e].x;
    const int pos = atomicAdd(p.sl_kcnt + list_kid(p, b, kvh, key), 1);
    p.sl_tr[pos] = slot0 + e;
  }
}

// One warp per key: sort the key's slots, then four groups of eight lanes take
// every fourth entry (each lane HD / 8 columns), and the groups' sums are
// combined in a fixed order.
template <int HD, bool BF16>
__global__ void __launch_bounds__(256) key_dkdv_kernel(const AttnParams p) {
  if (*p.sl_flag != 0) return;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int DL = HD / 8;  // columns per lane
  constexpr int NV = DL / 8;  // 16-byte vectors per lane and row
  __shared__ int sbuf[8][kKeyMaxEntries];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t kid = (int64_t)blockIdx.x * 8 + warp;
  if (kid >= p.sl_nk) return;
  const bool varlen = p.cu_k != nullptr;
  const int64_t lk = varlen ? p.rows_k : p.len_k;
  const int64_t tok = kid % lk;
  const int kvh = (int)((kid / lk) % p.hkv);
  const int b = varlen ? 0 : (int)(kid / lk / p.hkv);
  const int off = p.sl_koff[kid];
  const int n = p.sl_koff[kid + 1] - off;
  if (n > kKeyMaxEntries) return;  // a long key: key_long_kernel
  int* seg = p.sl_tr + off;

  // sort the segment by slot number
  if (n > 1 && n <= 32) {
    int x = lane < n ? seg[lane] : INT_MAX;
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1) {
        const int y = __shfl_xor_sync(0xffffffffu, x, j);
        const bool up = (lane & k) == 0, lower = (lane & j) == 0;
        x = (lower == up) ? min(x, y) : max(x, y);
      }
    }
    if (lane < n) seg[lane] = x;
    __syncwarp();
  } else if (n > 32) {
    int* a = sbuf[warp];
    for (int e = lane; e < n; e += 32) a[e] = seg[e];
    __syncwarp();
    for (int e = lane; e < n; e += 32) {
      const int x = a[e];
      int rank = 0;
      for (int f = 0; f < n; ++f) rank += a[f] < x ? 1 : 0;
      seg[rank] = x;
    }
    __syncwarp();
  }

  const int grp = lane >> 3, c0 = (lane & 7) * DL;
  float dk[DL], dv[DL];
#pragma unroll
  for (int x = 0; x < DL; ++x) dk[x] = dv[x] = 0.f;
  auto row_ptr = [&](int slot, const void* base, int64_t sb, int64_t sh, int64_t st) -> const uint4* {
    const int64_t hr = slot / kSupSlots;
    const int h = (int)(hr / p.rows_total);
    const int r = (int)(hr - (int64_t)h * p.rows_total);
    const int rb = varlen ? 0 : r / p.len_q;
    const int64_t tq = varlen ? r : r % p.len_q;
    return reinterpret_cast<const uint4*>(static_cast<const T*>(base) + (int64_t)rb * sb + (int64_t)h * sh +
                                          tq * st + c0);
  };
  for (int e = grp; e < n; e += 4) {
    const int slot = seg[e];
    const float pv = __int_as_float(p.sl_ent[slot].y);
    const float ds = p.sl_g[slot];
    const uint4* qp = row_ptr(slot, p.q, p.q_sb, p.q_sh, p.q_st);
    const uint4* dp = row_ptr(slot, p.dout, p.do_sb, p.do_sh, p.do_st);
    uint4 qv[NV], dv4[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      qv[v] = __ldg(qp + v);
      dv4[v] = __ldg(dp + v);
    }
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float f[8], g[8];
      unpack8<BF16>(qv[v], f);
      unpack8<BF16>(dv4[v], g);
#pragma unroll
      for (int x = 0; x < 8; ++x) {
        dk[v * 8 + x] = fmaf(ds, f[x], dk[v * 8 + x]);
        dv[v * 8 + x] = fmaf(pv, g[x], dv[v * 8 + x]);
      }
    }
  }
  // groups 0+1 and 2+3, then the two halves
#pragma unroll
  for (int x = 0; x < DL; ++x) {
    dk[x] += __shfl_xor_sync(0xffffffffu, dk[x], 8);
    dv[x] += __shfl_xor_sync(0xffffffffu, dv[x], 8);
    dk[x] += __shfl_xor_sync(0xffffffffu, dk[x], 16);
    dv[x] += __shfl_xor_sync(0xffffffffu, dv[x], 16);
  }
  if (grp != 0) return;
  const int64_t ko = varlen ? 0 : (int64_t)b;
  uint4* kd = reinterpret_cast<uint4*>(static_cast<T*>(p.dk) + ko * p.dk_sb + (int64_t)kvh * p.dk_sh + tok * p.dk_st + c0);
  uint4* vd = reinterpret_cast<uint4*>(static_cast<T*>(p.dv) + ko * p.dv_sb + (int64_t)kvh * p.dv_sh + tok * p.dv_st + c0);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    uint4 a, c;
    a.x = pack_pair<BF16>(dk[v * 8 + 0] * p.scale, dk[v * 8 + 1] * p.scale);
    a.y = pack_pair<BF16>(dk[v * 8 + 2] * p.scale, dk[v * 8 + 3] * p.scale);
    a.z = pack_pair<BF16>(dk[v * 8 + 4] * p.scale, dk[v * 8 + 5] * p.scale);
    a.w = pack_pair<BF16>(dk[v * 8 + 6] * p.scale, dk[v * 8 + 7] * p.scale);
    c.x = pack_pair<BF16>(dv[v * 8 + 0], dv[v * 8 + 1]);
    c.y = pack_pair<BF16>(dv[v * 8 + 2], dv[v * 8 + 3]);
    c.z = pack_pair<BF16>(dv[v * 8 + 4], dv[v * 8 + 5]);
    c.w = pack_pair<BF16>(dv[v * 8 + 6], dv[v * 8 + 7]);
    kd[v] = a;
    vd[v] = c;
  }
}

// Long keys (more than kKeyMaxEntries entries: attention sinks), one CTA per
// key at a time.  The rows holding the key are marked in a shared-memory
// bitmap over (query head of the group, row of the key's sequence), which
// orders them without a sort; the 16 warps take fixed contiguous ranges of the
// bitmap, each warp's four 8-lane groups take every fourth marked row in
// order, find the key in the row's sub-lists, and the partial sums are added
// in warp order, so the result is the same on every run.  A key whose
// sequence needs a larger bitmap sets kListKeyOverflow (the tile dK/dV kernel
// then recomputes every key).
constexpr int kLongThreads = 512;
constexpr int kLongWarps = kLongThreads / 32;
constexpr int kLongBitWords = 16384;  // 524288 (head, row) pairs

template <int HD>
constexpr size_t long_smem_bytes() { return (size_t)kLongBitWords * 4 + (size_t)kLongWarps * 2 * HD * 4; }

template <int HD, bool BF16>
__global__ void __launch_bounds__(kLongThreads) key_long_kernel(const AttnParams p) {
  if (*p.sl_flag != 0) return;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int DL = HD / 8, NV = DL / 8, NWG = HD / 32, LW = kSupSlots / NWG;
  extern __shared__ uint32_t lsm[];
  uint32_t* bits = lsm;
  float* parts = reinterpret_cast<float*>(lsm + kLongBitWords);  // [warp][dk, dv][HD]
  const int nlong = min(*(volatile int*)p.sl_long, p.sl_long_cap);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane >> 3, l8 = lane & 7, c0 = l8 * DL;
  const unsigned gmask = 0xffu << (grp * 8);
  const int G = p.hq / p.hkv;
  const bool varlen = p.cu_k != nullptr;
  const int64_t lk = varlen ? p.rows_k : p.len_k;
  for (int li = blockIdx.x; li < nlong; li += gridDim.x) {
    const int64_t kid = p.sl_long[1 + li];
    const int tok = (int)(kid % lk);
    const int kvh = (int)((kid / lk) % p.hkv);
    const int b = varlen ? 0 : (int)(kid / lk / p.hkv);
    int rlo, rn;  // the rows of the key's sequence
    if (!varlen) {
      rlo = b * p.len_q;
      rn = p.len_q;
    } else {
      int lo = 0, hi = p.batch - 1;  // the last sequence whose first key is <= tok
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.cu_k[mid] <= tok) lo = mid; else hi = mid - 1;
      }
      rlo = p.cu_q[lo];
      rn = p.cu_q[lo + 1] - rlo;
    }
    const int64_t nbits = (int64_t)G * rn;
    if (nbits > (int64_t)kLongBitWords * 32) {
      if (tid == 0) atomicOr(p.sl_flag, kListKeyOverflow);
      continue;
    }
    const int words = (int)((nbits + 31) / 32);
    for (int w = tid; w < words; w += kLongThreads) bits[w] = 0u;
    __syncthreads();
    const int off = p.sl_koff[kid], n = p.sl_koff[kid + 1] - off;
    for (int e = tid; e < n; e += kLongThreads) {
      const int slot = p.sl_tr[off + e];
      const int64_t hr = slot / kSupSlots;
      const int h = (int)(hr / p.rows_total);
      const int r = (int)(hr - (int64_t)h * p.rows_total);
      const int bit = (h - kvh * G) * rn + (r - rlo);
      atomicOr(&bits[bit >> 5], 1u << (bit & 31));
    }
    __syncthreads();
    float dk[DL], dv[DL];
#pragma unroll
    for (int x = 0; x < DL; ++x) dk[x] = dv[x] = 0.f;
    const int per = (words + kLongWarps - 1) / kLongWarps;
    int w = min(words, warp * per);
    const int wend = min(words, w + per);
    uint32_t m = w < wend ? bits[w] : 0u;
    for (;;) {
      // the next four marked rows of this warp's range, one per group (uniform)
      int idx[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        while (m == 0u && w + 1 < wend) m = bits[++w];
        if (m == 0u) {
          idx[k] = -1;
        } else {
          idx[k] = w * 32 + __ffs(m) - 1;
          m &= m - 1u;
        }
      }
      if (idx[0] < 0) break;
      const int mine = idx[grp];
      if (mine >= 0) {
        const int h = kvh * G + mine / rn;
        const int r = rlo + mine % rn;
        const int64_t hr = (int64_t)h * p.rows_total + r;
        // the key's slot in the row's sub-lists
        int slot = -1;
        for (int sw = 0; sw < NWG && slot < 0; ++sw) {
          const int c = p.sl_cnt[hr * NWG + sw];
          for (int e0 = 0; e0 < c && slot < 0; e0 += 8) {
            const int e = e0 + l8;
            const int64_t sl = hr * kSupSlots + sw * LW + e;
            const bool hit = e < c && p.sl_ent[sl].x == tok;
            const unsigned bal = __ballot_sync(gmask, hit) & gmask;
            if (bal) slot = __shfl_sync(gmask, (int)sl, __ffs(bal) - 1);
          }
        }
        if (slot >= 0) {
          const float pv = __int_as_float(p.sl_ent[slot].y);
          const float ds = p.sl_g[slot];
          const int rb = varlen ? 0 : r / p.len_q;
          const int64_t tq = varlen ? r : r % p.len_q;
          const uint4* qp = reinterpret_cast<const uint4*>(static_cast<const T*>(p.q) + (int64_t)rb * p.q_sb +
                                                           (int64_t)h * p.q_sh + tq * p.q_st + c0);
          const uint4* dp = reinterpret_cast<const uint4*>(static_cast<const T*>(p.dout) + (int64_t)rb * p.do_sb +
                                                           (int64_t)h * p.do_sh + tq * p.do_st + c0);
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            float f[8], g[8];
            unpack8<BF16>(__ldg(qp + v), f);
            unpack8<BF16>(__ldg(dp + v), g);
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              dk[v * 8 + x] = fmaf(ds, f[x], dk[v * 8 + x]);
              dv[v * 8 + x] = fmaf(pv, g[x], dv[v * 8 + x]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int x = 0; x < DL; ++x) {
      dk[x] += __shfl_xor_sync(0xffffffffu, dk[x], 8);
      dv[x] += __shfl_xor_sync(0xffffffffu, dv[x], 8);
      dk[x] += __shfl_xor_sync(0xffffffffu, dk[x], 16);
      dv[x] += __shfl_xor_sync(0xffffffffu, dv[x], 16);
    }
    if (grp == 0) {
#pragma unroll
      for (int x = 0; x < DL; ++x) {
        parts[(warp * 2 + 0) * HD + c0 + x] = dk[x];
        parts[(warp * 2 + 1) * HD + c0 + x] = dv[x];
      }
    }
    __syncthreads();
    if (tid < 2 * HD) {
      const int which = tid / HD, d = tid % HD;
      float acc = 0.f;
      for (int wp = 0; wp < kLongWarps; ++wp) acc += parts[(wp * 2 + which) * HD + d];
      const int64_t ko = varlen ? 0 : (int64_t)b;
      if (which == 0)
        static_cast<T*>(p.dk)[ko * p.dk_sb + (int64_t)kvh * p.dk_sh + (int64_t)tok * p.dk_st + d] =
            from_f32<T>(acc * p.scale);
      else
        static_cast<T*>(p.dv)[ko * p.dv_sb + (int64_t)kvh * p.dv_sh + (int64_t)tok * p.dv_st + d] = from_f32<T>(acc);
    }
    __syncthreads();  // bits and parts are reused by the next key
  }
}

template <int HD, bool BF16>
cudaError_t launch_list_bwd(const AttnParams& p, cudaStream_t s) {
  cudaError_t e = cudaMemsetAsync(p.sl_kcnt, 0, (size_t)p.sl_nk * sizeof(int), s);
  if (e != cudaSuccess) return e;
  const dim3 grid((p.rows_total + kRowsPerBlock - 1) / kRowsPerBlock, p.hq);
  if (p.norm == HFAN_SPARSEMAX)
    sparse_dq_kernel<HD, BF16, HFAN_SPARSEMAX><<<grid, 256, 0, s>>>(p);
  else
    sparse_dq_kernel<HD, BF16, HFAN_ENTMAX15><<<grid, 256, 0, s>>>(p);
  const unsigned nb = (unsigned)sparse_key_blocks(p.sl_nk);
  key_block_sum_kernel<<<nb, 256, 0, s>>>(p);
  key_scan_kernel<<<nb, 256, 0, s>>>(p);
  const int64_t subs = (int64_t)p.hq * p.rows_total * (HD / 32);
  key_fill_kernel<HD><<<(unsigned)((subs + 255) / 256), 256, 0, s>>>(p);
  key_dkdv_kernel<HD, BF16><<<(unsigned)((p.sl_nk + 7) / 8), 256, 0, s>>>(p);
  cudaError_t le = cudaFuncSetAttribute(key_long_kernel<HD, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)long_smem_bytes<HD>());
  if (le != cudaSuccess) return le;
  key_long_kernel<HD, BF16><<<(unsigned)min(p.sl_long_cap, 296), kLongThreads, long_smem_bytes<HD>(), s>>>(p);
  return cudaGetLastError();
}

}  // namespace

// dQ, the row correction, dK and dV from the support lists.  Every kernel
// reads the overflow flags on the device and returns at once when its tile
// counterpart has to run instead.  16-bit inputs and gradients, head_dim 64
// or 128.
cudaError_t sparse_list_bwd(int dtype, const AttnParams& p, cudaStream_t s) {
  const bool bf16 = dtype == HFAN_BFLOAT16;
  if (p.d == 128) return bf16 ? launch_list_bwd<128, true>(p, s) : launch_list_bwd<128, false>(p, s);
  return bf16 ? launch_list_bwd<64, true>(p, s) : launch_list_bwd<64, false>(p, s);
}

}  // namespace hfan
