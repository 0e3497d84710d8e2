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
//   tau      per (sequence, query head): the scores above zmax - 1 (<= 4096)
//            are compacted into shared memory and tau is solved exactly
//            (bracket + closed form, common.cuh)
//   pv       per unit: p = (z - tau)_+^a; V rows are read only for keys with
//            p > 0 for some head of the group (zero-probability keys cost no
//            V traffic)
//   combine  O = sum over splits of the partial P V
//
// Row statistics use the same layout as the other attention kernels, so the
// general paged backward can consume them.
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "params.cuh"
#include "tc_common.cuh"

namespace hfan {
namespace {

constexpr int kChunk = 1024;   // keys per split
constexpr int kUnroll = 4;      // key rows in flight per lane group
constexpr int kMaxRow = 32768; // longest row the split decode serves (score workspace per row)

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

// Row maxima of the sparse scores, kept in the tau slots of the workspace
// until the tau kernel replaces them: floats mapped to unsigned integers in
// the same order (so atomicMax finds the largest), 0 = no score yet (the
// slots are zeroed before the scores kernel).
__device__ __forceinline__ unsigned ordered_bits(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_float(unsigned u) {
  if (u == 0u) return kNegInf;
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// ------------------------------------------------------------------ softmax1
// One CTA per (sequence, split) and one warp per KV head, so the 8 heads of a
// token -- one contiguous 2 KB stretch of the page -- are read together.
template <typename T, int D, int G>
__global__ void __launch_bounds__(256, 2) decode_sm1_split(AttnParams p, DecodeWs ws) {
  using LN = Lanes<D>;
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = seq_len_k(p, b);
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

// ---------------------------------------------------- softmax1, tiled path
// Same work unit and result as decode_sm1_split, restructured so that HBM,
// not instruction issue, bounds it:
//  * a producer warp streams blocks of kBlk tokens (every KV head) into a
//    kStagesDec-deep shared-memory ring with TMA tile loads (a 3-D tensor map
//    over (dim, token, head), 128-byte swizzle, completion on mbarriers), so
//    several blocks per SM are in flight;
//  * one consumer warp per KV head computes with mma.sync m16n8k16 (the G
//    query heads padded to 16 rows): S = Q K^T over the block, the online
//    softmax on the accumulator fragments, then O += P V with P taken
//    directly from the S fragments as the A operand.  K and V fragments come
//    from the swizzled tiles with ldmatrix (V transposed), conflict-free.
// A block never crosses a page (pages hold a multiple of kBlk tokens).
constexpr int kBlk = 16;        // tokens per block (the MMA k extent of P V)
constexpr int kStagesDec = 3;   // ring depth

struct BulkCtl {
  uint64_t full[kStagesDec], empty[kStagesDec];
  int valid[kStagesDec];
  int abort;
};

// Bytes of one block of one cache (K or V): D/64 swizzled 64-dim halves of
// [hkv][kBlk] rows of 128 bytes.
template <int D>
__host__ __device__ constexpr uint32_t tiled_block_bytes(int hkv) {
  return (uint32_t)(D / 64) * 128u * kBlk * (uint32_t)hkv;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2_t(float a, float b) {
  return tc::pack2<std::is_same<T, __nv_bfloat16>::value>(a, b);
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(tc::smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(288, 1)
    decode_sm1_tiled(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, AttnParams p,
                     DecodeWs ws) {
  static_assert(G <= 8, "query heads per KV head");
  constexpr int NHALF = D / 64;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = seq_len_k(p, b);
  const int t0 = split * kChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kChunk);
  const int nblk = (t1 - t0 + kBlk - 1) / kBlk;
  const int hkv = p.hkv;  // <= 8 (host check)
  const uint32_t blk_bytes = tiled_block_bytes<D>(hkv), half_bytes = blk_bytes / NHALF;
  uint8_t* kring = dsm;
  uint8_t* vring = dsm + kStagesDec * blk_bytes;
  BulkCtl* ctl = reinterpret_cast<BulkCtl*>(dsm + 2 * kStagesDec * blk_bytes);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesDec; ++s) {
      tc::mbar_init(&ctl->full[s], 1);
      tc::mbar_init(&ctl->empty[s], hkv);
    }
    ctl->abort = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort_flag = &ctl->abort;
  const int* bt = page_row(p, b);

  if (warp == 8) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      tc::prefetch_tmap(&tm_k);
      tc::prefetch_tmap(&tm_v);
      for (int blk = 0; blk < nblk; ++blk) {
        const int s = blk % kStagesDec;
        if (blk >= kStagesDec &&
            !tc::mbar_wait(&ctl->empty[s], ((blk / kStagesDec) - 1) & 1, abort_flag)) {
          ctl->abort = 1;
          if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
          break;
        }
        const int t = t0 + blk * kBlk;
        const int page = bt[t / p.page_size];
        const int64_t tok0 = (int64_t)page * p.page_size + (t % p.page_size);
        const bool ok = page >= 0 && tok0 + kBlk <= p.num_cache_tokens;
        ctl->valid[s] = ok ? 1 : 0;
        if (ok) {
          tc::mbar_arrive_expect_tx(&ctl->full[s], 2 * blk_bytes);
#pragma unroll
          for (int hh = 0; hh < NHALF; ++hh) {
            tma_load_3d(tc::smem_u32(kring + s * blk_bytes + hh * half_bytes), &tm_k, &ctl->full[s], 64 * hh,
                        (int)tok0, 0);
            tma_load_3d(tc::smem_u32(vring + s * blk_bytes + hh * half_bytes), &tm_v, &ctl->full[s], 64 * hh,
                        (int)tok0, 0);
          }
        } else {
          if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevBadPage);
          tc::mbar_arrive(&ctl->full[s]);
        }
      }
    }
  } else if (warp < hkv) {
    // ---------------------------------------------------------- consumers
    const int kvh = warp;
    const int g = lane >> 2, tq = lane & 3;  // fragment row (query head) and column pair
    const float zs = p.scale * kLog2e;
    // A fragments of Q (rows >= G are zero): a0 = Q[g][16ks + 2tq ..], a2 = Q[g][16ks + 8 + 2tq ..]
    uint32_t qa[D / 16][2];
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) qa[ks][0] = qa[ks][1] = 0u;
    if (g < G) {
      const T* qr = static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)(kvh * G + g) * p.q_sh;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * tq);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 8 + 2 * tq);
      }
    }
    float o[D / 8][4];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m = kNegInf, l = 0.f;
    // ldmatrix row addresses of this lane: matrix mi = lane >> 3, row ri = lane & 7 (= token & 7,
    // which is also the 128-byte swizzle phase of the row)
    const int mi = lane >> 3, ri = lane & 7;
    for (int blk = 0; blk < nblk; ++blk) {
      const int s = blk % kStagesDec;
      bool got = tc::mbar_wait(&ctl->full[s], (blk / kStagesDec) & 1, abort_flag);
      got = __all_sync(0xffffffffu, got);
      if (!got) {
        if (lane == 0) {
          ctl->abort = 1;
          if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
        }
        break;
      }
      const bool bvalid = ctl->valid[s] != 0;
      const uint32_t kst = tc::smem_u32(kring + s * blk_bytes), vst = tc::smem_u32(vring + s * blk_bytes);
      // ---- S = Q K^T: two n-tiles of 8 tokens
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        // matrix mi: tokens 8 (mi >> 1) + ri, dims 16 ks + 8 (mi & 1) .. + 8
        const int dim0 = 16 * ks + 8 * (mi & 1);
        const int row = kvh * kBlk + 8 * (mi >> 1) + ri;
        const uint32_t addr = kst + (dim0 >> 6) * half_bytes + row * 128 + ((((dim0 & 63) >> 3) ^ ri) << 4);
        uint32_t kb4[4];
        ldsm_x4(addr, kb4);
        const uint32_t a[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
        mma16816<T>(sacc[0], a, kb4[0], kb4[1]);
        mma16816<T>(sacc[1], a, kb4[2], kb4[3]);
      }
      // ---- online softmax of row g over the block's 16 tokens (4 per lane)
      const int tb = t0 + blk * kBlk;
      float sv[4] = {sacc[0][0] * zs, sacc[0][1] * zs, sacc[1][0] * zs, sacc[1][1] * zs};
#pragma unroll
      for (int x = 0; x < 4; ++x) {
        const int tok = 8 * (x >> 1) + 2 * tq + (x & 1);
        if (!(bvalid && tb + tok < t1)) sv[x] = kNegInf;
      }
      float bmax = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 1));
      bmax = fmaxf(bmax, __shfl_xor_sync(0xffffffffu, bmax, 2));
      // lazy reference: move it only when the block max exceeds it by 2^8
      const bool move = bmax > m + 8.f;
      const float m_new = move ? bmax : m;
      const float alpha = move ? exp2f(m - m_new) : 1.f;  // 0 when m was -inf
      if (__any_sync(0xffffffffu, move)) {
        l *= alpha;
#pragma unroll
        for (int j = 0; j < D / 8; ++j) {
          o[j][0] *= alpha;
          o[j][1] *= alpha;
        }
      }
      m = m_new;
      float pv[4];
#pragma unroll
      for (int x = 0; x < 4; ++x) pv[x] = sv[x] > kNegInf ? exp2f(sv[x] - m) : 0.f;
      l += (pv[0] + pv[1]) + (pv[2] + pv[3]);
      uint32_t pa[4];
      pa[0] = pack2_t<T>(pv[0], pv[1]);
      pa[1] = 0u;
      pa[2] = pack2_t<T>(pv[2], pv[3]);
      pa[3] = 0u;
      // ---- O += P V: D/8 n-tiles of 8 dims, k = the block's 16 tokens
#pragma unroll
      for (int jp = 0; jp < D / 16; ++jp) {
        // matrix mi: dims 8 (2 jp + (mi >> 1)) .. + 8, tokens 8 (mi & 1) + ri (transposed load)
        const int dt = 2 * jp + (mi >> 1);
        const int row = kvh * kBlk + 8 * (mi & 1) + ri;
        const uint32_t addr = vst + (dt >> 3) * half_bytes + row * 128 + (((dt & 7) ^ ri) << 4);
        uint32_t vb4[4];
        ldsm_x4_t(addr, vb4);
        mma16816<T>(o[2 * jp], pa, vb4[0], vb4[1]);
        mma16816<T>(o[2 * jp + 1], pa, vb4[2], vb4[3]);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&ctl->empty[s]);
    }
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (g < G) {
      const int64_t unit = ((int64_t)b * p.hkv + kvh) * ws.splits + split;
      float* dst = ws.acc + (unit * G + g) * D + 2 * tq;
#pragma unroll
      for (int j = 0; j < D / 8; ++j) *reinterpret_cast<float2*>(dst + 8 * j) = make_float2(o[j][0], o[j][1]);
      if (tq == 0) {
        ws.ml[(unit * G + g) * 2 + 0] = m;
        ws.ml[(unit * G + g) * 2 + 1] = l;
      }
    }
  }
}

// Sparse scores through the same ring (K blocks only): z = s * zs for every
// key, written to the workspace rows like decode_sparse_scores.
template <typename T, int D, int G, int NORM>
__global__ void __launch_bounds__(288, 1)
    decode_sparse_scores_tiled(const __grid_constant__ CUtensorMap tm_k, AttnParams p, DecodeWs ws, int max_len) {
  static_assert(G <= 8, "query heads per KV head");
  constexpr int NHALF = D / 64;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = seq_len_k(p, b);
  const int t0 = split * kChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kChunk);
  const int nblk = (t1 - t0 + kBlk - 1) / kBlk;
  const int hkv = p.hkv;
  const uint32_t blk_bytes = tiled_block_bytes<D>(hkv), half_bytes = blk_bytes / NHALF;
  constexpr int NS = 2 * kStagesDec;  // K only: twice the stages in the same space
  uint8_t* kring = dsm;
  BulkCtl* ctl0 = reinterpret_cast<BulkCtl*>(dsm + NS * blk_bytes);
  BulkCtl* ctl1 = ctl0 + 1;
  auto full = [&](int s_) { return s_ < kStagesDec ? &ctl0->full[s_] : &ctl1->full[s_ - kStagesDec]; };
  auto empty = [&](int s_) { return s_ < kStagesDec ? &ctl0->empty[s_] : &ctl1->empty[s_ - kStagesDec]; };
  auto valid = [&](int s_) -> int* { return s_ < kStagesDec ? &ctl0->valid[s_] : &ctl1->valid[s_ - kStagesDec]; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s_ = 0; s_ < NS; ++s_) {
      tc::mbar_init(full(s_), 1);
      tc::mbar_init(empty(s_), hkv);
    }
    ctl0->abort = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  volatile int* abort_flag = &ctl0->abort;
  const int* bt = page_row(p, b);

  if (warp == 8) {
    if (lane == 0) {
      tc::prefetch_tmap(&tm_k);
      for (int blk = 0; blk < nblk; ++blk) {
        const int s_ = blk % NS;
        if (blk >= NS && !tc::mbar_wait(empty(s_), ((blk / NS) - 1) & 1, abort_flag)) {
          ctl0->abort = 1;
          if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
          break;
        }
        const int t = t0 + blk * kBlk;
        const int page = bt[t / p.page_size];
        const int64_t tok0 = (int64_t)page * p.page_size + (t % p.page_size);
        const bool ok = page >= 0 && tok0 + kBlk <= p.num_cache_tokens;
        *valid(s_) = ok ? 1 : 0;
        if (ok) {
          tc::mbar_arrive_expect_tx(full(s_), blk_bytes);
#pragma unroll
          for (int hh = 0; hh < NHALF; ++hh)
            tma_load_3d(tc::smem_u32(kring + s_ * blk_bytes + hh * half_bytes), &tm_k, full(s_), 64 * hh, (int)tok0,
                        0);
        } else {
          if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevBadPage);
          tc::mbar_arrive(full(s_));
        }
      }
    }
  } else if (warp < hkv) {
    const int kvh = warp;
    const int g = lane >> 2, tq = lane & 3;
    const float zs = NORM == HFAN_SPARSEMAX ? p.scale : 0.5f * p.scale;
    uint32_t qa[D / 16][2];
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) qa[ks][0] = qa[ks][1] = 0u;
    if (g < G) {
      const T* qr = static_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)(kvh * G + g) * p.q_sh;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        qa[ks][0] = *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 2 * tq);
        qa[ks][1] = *reinterpret_cast<const uint32_t*>(qr + 16 * ks + 8 + 2 * tq);
      }
    }
    float* srow = ws.scores + ((int64_t)b * p.hq + kvh * G + (g < G ? g : 0)) * max_len;
    float zmax = kNegInf;
    const int mi = lane >> 3, ri = lane & 7;
    for (int blk = 0; blk < nblk; ++blk) {
      const int s_ = blk % NS;
      bool got = tc::mbar_wait(full(s_), (blk / NS) & 1, abort_flag);
      got = __all_sync(0xffffffffu, got);
      if (!got) {
        if (lane == 0) {
          ctl0->abort = 1;
          if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
        }
        break;
      }
      const bool bvalid = *valid(s_) != 0;
      const uint32_t kst = tc::smem_u32(kring + s_ * blk_bytes);
      float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int dim0 = 16 * ks + 8 * (mi & 1);
        const int row = kvh * kBlk + 8 * (mi >> 1) + ri;
        const uint32_t addr = kst + (dim0 >> 6) * half_bytes + row * 128 + ((((dim0 & 63) >> 3) ^ ri) << 4);
        uint32_t kb4[4];
        ldsm_x4(addr, kb4);
        const uint32_t a[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
        mma16816<T>(sacc[0], a, kb4[0], kb4[1]);
        mma16816<T>(sacc[1], a, kb4[2], kb4[3]);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(empty(s_));
      const int tb = t0 + blk * kBlk;
      if (g < G && bvalid) {
#pragma unroll
        for (int x = 0; x < 4; ++x) {
          const int t = tb + 8 * (x >> 1) + 2 * tq + (x & 1);
          if (t < t1) {
            const float z = sacc[x >> 1][x & 1] * zs;
            srow[t] = z;
            zmax = fmaxf(zmax, z);
          }
        }
      }
    }
    // the four lanes of a head hold its keys: one atomic per head and CTA
    zmax = fmaxf(zmax, __shfl_xor_sync(0xffffffffu, zmax, 1));
    zmax = fmaxf(zmax, __shfl_xor_sync(0xffffffffu, zmax, 2));
    if (g < G && tq == 0 && zmax > kNegInf)
      atomicMax(reinterpret_cast<unsigned*>(ws.tau) + (int64_t)b * p.hq + kvh * G + g, ordered_bits(zmax));
  }
}

// Tensor map over one cache, dims (D, tokens, Hkv) with the cache's token and
// head strides, box (64, kBlk, Hkv), 128-byte swizzle.
inline bool make_cache_map(CUtensorMap* m, const void* base, bool bf16, int d, int64_t tokens, int hkv,
                           int64_t st, int64_t sh) {
  auto fn = tc::encode_fn();
  if (fn == nullptr) return false;
  cudaFree(nullptr);  // a current context for the driver-side encoder (see tc::make_map)
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)tokens, (cuuint64_t)hkv};
  cuuint64_t strides[2] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)kBlk, (cuuint32_t)hkv};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The tiled path applies: at most 8 KV heads, pages of a multiple of kBlk
// tokens, a ring that fits, and both caches describable by a tensor map.
template <typename T, int D>
bool tiled_ok(const AttnParams& p, CUtensorMap* mk, CUtensorMap* mv) {
  if (p.hkv > 8 || p.page_size % kBlk) return false;
  if (p.num_cache_tokens >= ((int64_t)1 << 31)) return false;
  if (2 * kStagesDec * (size_t)tiled_block_bytes<D>(p.hkv) + sizeof(BulkCtl) + 1024 > 220 * 1024) return false;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  return make_cache_map(mk, p.k, bf16, D, p.num_cache_tokens, p.hkv, p.k_st, p.k_sh) &&
         make_cache_map(mv, p.v, bf16, D, p.num_cache_tokens, p.hkv, p.v_st, p.v_sh);
}

template <typename T, int D, int G>
__global__ void decode_sm1_combine(AttnParams p, DecodeWs ws) {
  const int b = blockIdx.y, hq = blockIdx.x;
  const int kvh = hq / G, h = hq % G;
  const int L = seq_len_k(p, b);
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
  const int L = seq_len_k(p, b);
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
    float zmax = kNegInf;  // of head li (lanes li < G write head li's scores)
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
          if (valid[u] && li == h % LN::LPT) {
            srow[(int64_t)h * max_len + t] = sv;
            zmax = fmaxf(zmax, sv);
          }
        }
      }
    }
    if (li < G && zmax > kNegInf)
      atomicMax(reinterpret_cast<unsigned*>(ws.tau) + (int64_t)b * p.hq + kvh * G + li, ordered_bits(zmax));
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

// One CTA per (sequence, query head): exact tau of the score row.
// tau >= zmax - 1, so only the scores above zmax - 1 matter (zmax comes from
// the scores kernel).  One pass over the row, coalesced with four keys per
// thread in flight, compacts the candidates into a shared-memory list in index
// order (per step of 2048 keys: a ballot per warp and quarter, one scan of the
// 64 counts).  All 16 warps then iterate the solve on the list, the four sums
// reduced across the block in a fixed order, so tau is the same on every run.
// Rows with more candidates than the list holds iterate over the whole row in
// global memory.
constexpr int kTauCand = 4096;
constexpr int kTauThreads = 512;
constexpr int kTauWarps = kTauThreads / 32;
constexpr int kTauVec = 4;  // keys per thread and step (loads in flight; 8 measured slower)

template <int NORM>
__global__ void __launch_bounds__(kTauThreads) decode_sparse_tau(AttnParams p, DecodeWs ws, int max_len) {
  __shared__ float red[32];
  __shared__ float cand[kTauCand];
  __shared__ int qcount[kTauVec * kTauWarps];  // per step: candidates of (part, warp), then their offsets
  __shared__ float part[2][kTauWarps][4];
  __shared__ int s_total;
  const int b = blockIdx.y, hq = blockIdx.x;
  const int L = seq_len_k(p, b);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* zrow = ws.scores + ((int64_t)b * p.hq + hq) * max_len;
  constexpr int STEP = kTauVec * kTauThreads;
  // the row maximum, left in this row's tau slot by the scores kernel
  const float zmax = ordered_float(reinterpret_cast<const unsigned*>(ws.tau)[(int64_t)b * p.hq + hq]);
  __syncthreads();  // every thread has read the slot before thread 0 overwrites it
  float tau = kPosInf, support = 0.f;
  if (zmax > kNegInf) {
    const float t0 = zmax - 1.f;
    if (tid == 0) s_total = 0;
    __syncthreads();
    for (int j0 = 0; j0 < L; j0 += STEP) {
      float x[kTauVec];
      unsigned bal[kTauVec];
#pragma unroll
      for (int k = 0; k < kTauVec; ++k) {
        const int j = j0 + k * kTauThreads + tid;
        x[k] = j < L ? zrow[j] : kNegInf;
      }
#pragma unroll
      for (int k = 0; k < kTauVec; ++k) {
        bal[k] = __ballot_sync(0xffffffffu, x[k] > t0);
        if (lane == 0) qcount[k * kTauWarps + warp] = __popc(bal[k]);
      }
      __syncthreads();
      if (warp == 0) {  // exclusive scan of the counts in (part, warp) order
        constexpr int PL = kTauVec * kTauWarps / 32;  // counts per lane
        int c[PL], sum = 0;
#pragma unroll
        for (int i = 0; i < PL; ++i) sum += (c[i] = qcount[PL * lane + i]);
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        int base = s_total + incl - sum;
        __syncwarp();  // every lane has read s_total
#pragma unroll
        for (int i = 0; i < PL; ++i) {
          qcount[PL * lane + i] = base;
          base += c[i];
        }
        if (lane == 31) s_total = base;
      }
      __syncthreads();
      const unsigned below = (1u << lane) - 1u;
#pragma unroll
      for (int k = 0; k < kTauVec; ++k) {
        if (x[k] > t0) {
          const int pos = qcount[k * kTauWarps + warp] + __popc(bal[k] & below);
          if (pos < kTauCand) cand[pos] = x[k];
        }
      }
      __syncthreads();  // qcount is rewritten by the next step
    }
    const int total = s_total;
    if (total <= kTauCand) {
      float t = t0, tr = kPosInf, sup = 0.f;
      for (int it = 0; it < 64; ++it) {
        TauStats st{0.f, 0.f, 0.f, kPosInf};
        for (int j = tid; j < total; j += kTauThreads) tau_accumulate(st, cand[j], t);
        st.cnt = warp_sum(st.cnt);
        st.s1 = warp_sum(st.s1);
        st.s2 = warp_sum(st.s2);
        st.zmin = warp_min(st.zmin);
        float* mine = part[it & 1][warp];
        if (lane == 0) {
          mine[0] = st.cnt;
          mine[1] = st.s1;
          mine[2] = st.s2;
          mine[3] = st.zmin;
        }
        __syncthreads();  // parts of this iteration complete; the other buffer is free
        TauStats all{0.f, 0.f, 0.f, kPosInf};
#pragma unroll
        for (int w = 0; w < kTauWarps; ++w) {
          const float* o = part[it & 1][w];
          all.cnt += o[0];
          all.s1 += o[1];
          all.s2 += o[2];
          all.zmin = fminf(all.zmin, o[3]);
        }
        sup = all.cnt;
        if (tau_step(NORM, all, &t, &tr)) break;  // uniform: every thread holds the same sums
      }
      tau = tr;
      support = sup;
    } else {
      float t = t0;
      for (int it = 0; it < 64; ++it) {
        TauStats st{0.f, 0.f, 0.f, kPosInf};
        for (int j = tid; j < L; j += blockDim.x) tau_accumulate(st, zrow[j], t);
        st.cnt = block_sum(st.cnt, red);
        st.s1 = block_sum(st.s1, red);
        st.s2 = block_sum(st.s2, red);
        st.zmin = block_min(st.zmin, red);
        support = st.cnt;
        if (tau_step(NORM, st, &t, &tau)) break;  // uniform: every thread sees the same sums
      }
    }
  }
  if (tid == 0) {
    ws.tau[(int64_t)b * p.hq + hq] = tau;
    const int64_t si = (int64_t)hq * p.rows_total + b;
    p.stats[si] = tau;
    p.stats[(int64_t)p.hq * p.rows_total + si] = support;
  }
}

// The warp reads the scores of 32 keys at a time (coalesced, every head of
// the group), ballots the keys with a nonzero probability for some head and
// reads V rows only for those; lane l accumulates head dims [D/32 l, D/32 (l+1)).
template <typename T, int D, int G, int NORM>
__global__ void __launch_bounds__(256) decode_sparse_pv(AttnParams p, DecodeWs ws, int max_len) {
  constexpr int DL = D / 32;  // dims per lane (4 or 2)
  const int b = blockIdx.y, split = blockIdx.x;
  const int L = seq_len_k(p, b);
  const int t0 = split * kChunk;
  if (t0 >= L) return;
  const int t1 = min(L, t0 + kChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int* bt = page_row(p, b);
  const T* vp = static_cast<const T*>(p.v);
  for (int kvh = warp; kvh < p.hkv; kvh += nwarps) {
    float tau[G];
#pragma unroll
    for (int h = 0; h < G; ++h) tau[h] = ws.tau[(int64_t)b * p.hq + kvh * G + h];
    const float* srow = ws.scores + ((int64_t)b * p.hq + kvh * G) * max_len;
    float acc[G][DL];
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int i = 0; i < DL; ++i) acc[h][i] = 0.f;
    for (int tb = t0; tb < t1; tb += 32) {  // warp-uniform bound (ballots, shuffles)
      const int t = tb + lane;
      float pr[G];
      bool any = false;
#pragma unroll
      for (int h = 0; h < G; ++h) {
        pr[h] = t < t1 ? sparse_prob(NORM, srow[(int64_t)h * max_len + t], tau[h]) : 0.f;
        any |= pr[h] > 0.f;
      }
      unsigned mask = __ballot_sync(0xffffffffu, any);
      while (mask) {
        const int src = __ffs(mask) - 1;
        mask &= mask - 1;
        float ps[G];
#pragma unroll
        for (int h = 0; h < G; ++h) ps[h] = __shfl_sync(0xffffffffu, pr[h], src);
        const int64_t tok = phys_token(p, bt, tb + src);
        if (tok < 0) continue;
        const T* vr = vp + tok * p.v_st + (int64_t)kvh * p.v_sh + lane * DL;
        float vx[DL];
        if constexpr (DL == 4) {
          const uint2 u = *reinterpret_cast<const uint2*>(vr);
          const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
          for (int i = 0; i < 4; ++i) vx[i] = to_f32<T>(e[i]);
        } else {
          const uint32_t u = *reinterpret_cast<const uint32_t*>(vr);
          const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
          for (int i = 0; i < DL; ++i) vx[i] = to_f32<T>(e[i]);
        }
#pragma unroll
        for (int h = 0; h < G; ++h)
#pragma unroll
          for (int i = 0; i < DL; ++i) acc[h][i] = fmaf(ps[h], vx[i], acc[h][i]);
      }
    }
    const int64_t unit = ((int64_t)b * p.hkv + kvh) * ws.splits + split;
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int i = 0; i < DL; ++i) ws.acc[(unit * G + h) * D + lane * DL + i] = acc[h][i];
  }
}

template <typename T, int D, int G>
__global__ void decode_sparse_combine(AttnParams p, DecodeWs ws) {
  const int b = blockIdx.y, hq = blockIdx.x;
  const int kvh = hq / G, h = hq % G;
  const int ns = (seq_len_k(p, b) + kChunk - 1) / kChunk;
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

// Launches the tiled scores kernel when its conditions hold; false leaves the
// work to decode_sparse_scores.
template <typename T, int D, int G, int NORM>
bool launch_scores_tiled(const AttnParams& p, DecodeWs ws, int max_len, dim3 grid, cudaStream_t s) {
  CUtensorMap mk, mv;
  if (!tiled_ok<T, D>(p, &mk, &mv)) return false;
  const size_t smem = 2 * kStagesDec * (size_t)tiled_block_bytes<D>(p.hkv) + 2 * sizeof(BulkCtl) + 1024;
  if (cudaFuncSetAttribute(decode_sparse_scores_tiled<T, D, G, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return false;
  decode_sparse_scores_tiled<T, D, G, NORM><<<grid, 288, smem, s>>>(mk, p, ws, max_len);
  return true;
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
    CUtensorMap mk, mv;
    if (tiled_ok<T, D>(p, &mk, &mv)) {
      const size_t smem = 2 * kStagesDec * (size_t)tiled_block_bytes<D>(p.hkv) + sizeof(BulkCtl) + 1024;
      cudaError_t e = cudaFuncSetAttribute(decode_sm1_tiled<T, D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem);
      if (e != cudaSuccess) return e;
      decode_sm1_tiled<T, D, G><<<grid_u, 288, smem, s>>>(mk, mv, p, ws);
    } else {
      decode_sm1_split<T, D, G><<<grid_u, ut, 0, s>>>(p, ws);
    }
    decode_sm1_combine<T, D, G><<<grid_r, D, 0, s>>>(p, ws);
    return cudaGetLastError();
  }
  // the row maxima of the scores kernels start at "no score" (see ordered_bits)
  cudaError_t e = cudaMemsetAsync(ws.tau, 0, (size_t)p.batch * p.hq * sizeof(float), s);
  if (e != cudaSuccess) return e;
  if (p.norm == HFAN_SPARSEMAX) {
    if (!launch_scores_tiled<T, D, G, HFAN_SPARSEMAX>(p, ws, max_len, grid_u, s))
      decode_sparse_scores<T, D, G, HFAN_SPARSEMAX><<<grid_u, ut, 0, s>>>(p, ws, max_len);
    decode_sparse_tau<HFAN_SPARSEMAX><<<grid_r, kTauThreads, 0, s>>>(p, ws, max_len);
    decode_sparse_pv<T, D, G, HFAN_SPARSEMAX><<<grid_u, ut, 0, s>>>(p, ws, max_len);
  } else {
    if (!launch_scores_tiled<T, D, G, HFAN_ENTMAX15>(p, ws, max_len, grid_u, s))
      decode_sparse_scores<T, D, G, HFAN_ENTMAX15><<<grid_u, ut, 0, s>>>(p, ws, max_len);
    decode_sparse_tau<HFAN_ENTMAX15><<<grid_r, kTauThreads, 0, s>>>(p, ws, max_len);
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
// point where they decode: code running on an inference server's hot path,
// and embedders that own the GPU allocator and
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
