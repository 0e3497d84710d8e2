// Tensor-core fused attention backward for 16-bit inputs on sm_100a.
//
// Two kernels with the forward's warp roles: HD / 32 row warpgroups (thread
// = TMEM lane = tile row), one TMA producer warp and two MMA issuer warps.
//
// dq kernel  (one CTA per 128 query rows of one (batch, query head))
//     per key tile:  S = Q K^T, dP = dO V^T          (TMEM, f32; issuer 1)
//                    dS = w (dP - c)                  (row warps -> TMEM, packed 16-bit)
//                    dQ += dS K                       (TMEM; issuer 2, K reused as an MN-major operand)
//     K streams through a 3-stage ring (it stays until its dQ MMA), V through
//     2 stages.  w = p for softmax1 (p = exp2(s log2e scale - m) / l from the
//     saved row statistics) and w = 1[p>0] (sparsemax) or sqrt(p) (entmax15):
//     the closed-form backwards of vutils/entmax.py:148-157 and :175-183 and
//     the softmax Jacobian.  The row correction c is sum_j w dP / sum_j w =
//     dO . wmean for the sparse normalizers (wmean = the w-weighted mean of V
//     saved by the forward; without it, a first pass over the key tiles) and
//     O . dO for softmax1 (the implicit sink has value 0).  c is saved for
//     the dk/dv kernel.
//
// dk/dv kernel  (one CTA per 128 keys of one (batch, KV head); it walks every
//                query head of the KV group, so GQA needs no atomics)
//     per unit (query head, 64 query rows):
//                      S^T = K Q^T, dP^T = V dO^T      (TMEM, double-buffered; issuer 1)
//                      P^T, dS^T                        (row warps -> shared memory, double-buffered)
//                      dV += P^T dO,  dK += dS^T Q      (TMEM accumulators; issuer 2)
//     Q / dO stream through a 3-stage ring of 64-row tiles.
//
// Sparse normalizers skip the key tiles (dq kernel) and units (dk/dv kernel)
// whose probabilities are all zero, from the forward's tile mask.  With the
// forward's support lists (sparsemax) both kernels return at once unless the
// overflow flag asks for them: sparse_bwd.cu computes the gradients from the
// lists.  Optional
// dropout scales dP by the forward's keep / (1 - p_drop) and feeds dV the
// dropped probabilities.  Gradients are written in the input dtype; dK
// carries the softmax scale.
#include "common.cuh"
#include "params.cuh"
#include "tc_common.cuh"
#include "tc_ptx.cuh"

namespace hfan {

cudaError_t sparse_list_bwd(int dtype, const AttnParams& p, cudaStream_t s);  // sparse_bwd.cu

namespace {

using namespace tc;

constexpr int kBM = 128;
constexpr int kBN = 128;

template <int NORM> __device__ __forceinline__ float zscale(float scale) {
  return NORM == HFAN_SOFTMAX1 ? scale * kLog2e : (NORM == HFAN_SPARSEMAX ? scale : 0.5f * scale);
}

// Weight w and probability p of one score (z units) given the row statistics.
template <int NORM>
__device__ __forceinline__ void weight(float z, float st0, float inv_l, float* w, float* pr) {
  if (NORM == HFAN_SOFTMAX1) {
    float e = ex2_ftz(z - st0) * inv_l;
    *w = e;
    *pr = e;
  } else {
    float d = z - st0;
    if (d > 0.f) {
      *w = NORM == HFAN_SPARSEMAX ? 1.f : d;
      *pr = NORM == HFAN_SPARSEMAX ? d : d * d;
    } else {
      *w = 0.f;
      *pr = 0.f;
    }
  }
}

// =========================================================== dq kernel
constexpr int kQStagesK = 3;  // K stays resident until its dQ MMA: one stage deeper than V
constexpr int kTileListMax = 512;  // key tiles a dQ CTA can skip over (65536 keys)
constexpr int kQStagesV = 2;

struct QBars {
  uint64_t qd_full;
  uint64_t k_full[kQStagesK], k_empty[kQStagesK], v_full[kQStagesV], v_empty[kQStagesV];
  uint64_t sdp_full, sdp_empty, ds_full[2], ds_empty[2], dq_done;
};

template <int HD>
struct QLayout {
  static constexpr int NH = HD / 64;
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t DO = Q + NH * kHalf;
  static constexpr uint32_t K = DO + NH * kHalf;
  static constexpr uint32_t V = K + kQStagesK * NH * kHalf;
  static constexpr uint32_t BARS = V + kQStagesV * NH * kHalf;
  static constexpr uint32_t CTL = BARS + sizeof(QBars);
  static constexpr uint32_t LIST = CTL + 16;                   // [kTileListMax] active key tiles, increasing
  static constexpr uint32_t TOTAL = LIST + kTileListMax * 2 + 1024;
};

template <int HD, bool BF16, int NORM, bool DROP>
__global__ void __launch_bounds__(Roles<HD, 2>::THREADS, 1)
    tc_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                     const AttnParams p) {
  // the support lists are complete: sparse_list_bwd computed dQ and c
  if (NORM != HFAN_SOFTMAX1 && p.sl_flag != nullptr && (*p.sl_flag & kListRowOverflow) == 0) return;
  using L = QLayout<HD>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int NH = L::NH;
  constexpr uint32_t TILE = NH * kHalf;
  constexpr bool SPARSE = NORM != HFAN_SOFTMAX1;
  // Sparse normalizers sweep the key tiles twice (the row correction c, then
  // dQ) unless the forward saved wmean, which gives c = dO . wmean directly.
  const int NPASS = SPARSE && p.wm == nullptr ? 2 : 1;
  constexpr uint32_t IDESC_S = idesc_f16(BF16, kBM, kBN, false, false);
  constexpr uint32_t IDESC_DQ = idesc_f16(BF16, kBM, HD, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  QBars* bars = reinterpret_cast<QBars*>(smem + L::BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::CTL);
  int* abort_ptr = reinterpret_cast<int*>(smem + L::CTL + 4);
  int* nact_ptr = reinterpret_cast<int*>(smem + L::CTL + 8);
  uint16_t* tlist = reinterpret_cast<uint16_t*>(smem + L::LIST);
  volatile int* abort_flag = abort_ptr;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint3 tile = tile_coords(p.tile_lpt);
  const int b = tile.z, h = tile.y;
  const int qt = gridDim.x - 1 - tile.x;
  const Geometry g = geometry(p, b);
  const int q0 = qt * kBM;
  if (q0 >= g.q_len) return;
  const int kvh = h / (p.hq / p.hkv);
  const bool varlen = p.cu_q != nullptr;
  const int qtok = varlen ? g.q_start + q0 : q0;
  const int ktok0 = varlen ? g.k_start : 0;
  const int bcoord = varlen ? 0 : b;

  const int last_row = min(q0 + kBM - 1, g.q_len - 1);
  int k_hi = g.k_len;
  if (p.causal) k_hi = min(k_hi, last_row + g.shift + 1);
  int k_lo = 0;
  if (p.window_left > 0) k_lo = max(0, q0 + g.shift - p.window_left + 1);
  k_lo = (k_lo / kBN) * kBN;
  const int n_tiles = k_hi > k_lo ? (k_hi - k_lo + kBN - 1) / kBN : 0;
  // Sparse normalizers skip the key tiles where every probability of the 128
  // rows is zero (no S, dP or dQ work: w = 0 there).  Warp 0 ORs the
  // forward's bits of the two 64-row blocks (lane = word) and writes the
  // active tiles, relative to k_lo, in increasing order to tlist.
  const int kt0 = k_lo / kBN;
  const bool use_mask = SPARSE && p.tile_mask != nullptr && kt0 + n_tiles <= kTileListMax;
  if (warp == 0) {
    uint32_t bits = 0u;
    if (use_mask && lane < p.mask_words) {
      const uint32_t* m = p.tile_mask + ((int64_t)(h * p.batch + b) * p.mask_qb + 2 * qt) * p.mask_words;
      bits = m[lane] | m[p.mask_words + lane];
      const int lo = kt0 - 32 * lane, hi = kt0 + n_tiles - 32 * lane;  // keep tiles [kt0, kt0 + n_tiles)
      if (lo > 0) bits = lo >= 32 ? 0u : bits & (~0u << lo);
      if (hi < 32) bits = hi <= 0 ? 0u : bits & (~0u >> (32 - hi));
    }
    const int c = __popc(bits);
    int pre = c;  // inclusive prefix sum over the lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, pre, o);
      if (lane >= o) pre += y;
    }
    const int total = __shfl_sync(0xffffffffu, pre, 31);
    int pos = pre - c;
    for (uint32_t rest = bits; rest != 0u; rest &= rest - 1u)
      tlist[pos++] = (uint16_t)(32 * lane + __ffs(rest) - 1 - kt0);
    if (lane == 0) *nact_ptr = use_mask ? total : n_tiles;
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->qd_full, 1);
    for (int s = 0; s < kQStagesK; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < kQStagesV; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->sdp_full, 1);
    mbar_init(&bars->sdp_empty, Roles<HD>::ROW_THREADS / 32);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->ds_full[s], Roles<HD>::ROW_THREADS / 32);
      mbar_init(&bars->ds_empty[s], 1);
    }
    mbar_init(&bars->dq_done, 1);
    *abort_ptr = 0;
    fence_barrier_init();
  }
  if (warp == Roles<HD>::MMA_WARP) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: S [0, 128), dP [128, 256), dQ [256, 256 + HD), dS double buffer
  // [384, 512) as packed 16-bit pairs (the A operand of the dQ MMA)
  const uint32_t tmem_s = tmem, tmem_dp = tmem + 128, tmem_dq = tmem + 256, tmem_ds = tmem + 384;
  // Active key tiles (relative index t, in increasing order): every role walks
  // the same list; ring stages and buffer parities count list positions.
  const int n_act = *nact_ptr;
  auto tile_at = [&](int a) -> int { return use_mask ? (int)tlist[a] : a; };

  if (warp == Roles<HD>::TMA_WARP) {
    if (lane == 0 && n_act > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_do);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&bars->qd_full, 2 * TILE);
      for (int hh = 0; hh < NH; ++hh) {
        tma_load_4d(smem + L::Q + hh * kHalf, &tm_q, &bars->qd_full, 64 * hh, qtok, h, bcoord);
        tma_load_4d(smem + L::DO + hh * kHalf, &tm_do, &bars->qd_full, 64 * hh, qtok, h, bcoord);
      }
      bool ok = true;
      uint32_t kc = 0;
      for (int pass = 0; pass < NPASS && ok; ++pass) {
        for (int a = 0; a < n_act && ok; ++a) {
          const int kb = k_lo + tile_at(a) * kBN;
          const int ks = kc % kQStagesK, vs = kc % kQStagesV;
          if (!(ok = mbar_wait(&bars->k_empty[ks], ((kc / kQStagesK) & 1) ^ 1, abort_flag))) break;
          mbar_arrive_expect_tx(&bars->k_full[ks], TILE);
          for (int hh = 0; hh < NH; ++hh)
            tma_load_4d(smem + L::K + ks * TILE + hh * kHalf, &tm_k, &bars->k_full[ks], 64 * hh, ktok0 + kb, kvh,
                        bcoord);
          if (!(ok = mbar_wait(&bars->v_empty[vs], ((kc / kQStagesV) & 1) ^ 1, abort_flag))) break;
          mbar_arrive_expect_tx(&bars->v_full[vs], TILE);
          for (int hh = 0; hh < NH; ++hh)
            tma_load_4d(smem + L::V + vs * TILE + hh * kHalf, &tm_v, &bars->v_full[vs], 64 * hh, ktok0 + kb, kvh,
                        bcoord);
          ++kc;
        }
      }
      if (!ok) {
        *abort_ptr = 1;
        if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
      }
    }
  } else if (warp == Roles<HD>::MMA_WARP) {
    // S and dP issuer (every pass).  dQ has its own issuer warp, so that the
    // waits of one overlap the tensor work of the other.
    if (lane == 0 && n_act > 0) {
      const uint32_t q_base = smem_u32(smem + L::Q), do_base = smem_u32(smem + L::DO);
      const uint32_t k_base = smem_u32(smem + L::K), v_base = smem_u32(smem + L::V);
      bool ok = mbar_wait(&bars->qd_full, 0, abort_flag);
      uint32_t kc = 0, sdc = 0;
      for (int pass = 0; pass < NPASS && ok; ++pass) {
        const bool last = pass == NPASS - 1;
        for (int a = 0; a < n_act && ok; ++a) {
          const int s = kc % kQStagesK, vs = kc % kQStagesV;
          if (!(ok = mbar_wait(&bars->k_full[s], (kc / kQStagesK) & 1, abort_flag))) break;
          if (!(ok = mbar_wait(&bars->v_full[vs], (kc / kQStagesV) & 1, abort_flag))) break;
          if (!(ok = mbar_wait(&bars->sdp_empty, (sdc & 1) ^ 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            mma_f16_ss(tmem_s, sw128_desc(q_base + off, 16, 1024), sw128_desc(k_base + s * TILE + off, 16, 1024),
                       IDESC_S, kk > 0);
          }
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kHalf + (kk & 3) * 32;
            mma_f16_ss(tmem_dp, sw128_desc(do_base + off, 16, 1024), sw128_desc(v_base + vs * TILE + off, 16, 1024),
                       IDESC_S, kk > 0);
          }
          mma_commit(&bars->sdp_full);
          mma_commit(&bars->v_empty[vs]);
          // K stays resident for dQ in the last pass (the dQ issuer releases it)
          if (!last) mma_commit(&bars->k_empty[s]);
          ++sdc;
          ++kc;
        }
      }
      if (!ok) {
        *abort_ptr = 1;
        if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
      }
    }
  } else if (warp == Roles<HD>::MMA2_WARP) {
    // dQ += dS K issuer (last pass).  K(t) sits in stage ((NPASS - 1) n + t) % 3;
    // it was loaded before S(t), which preceded dS(t).  dS(t) is read from
    // TMEM buffer t & 1.
    if (lane == 0 && n_act > 0) {
      const uint32_t k_base = smem_u32(smem + L::K);
      bool ok = true;
      for (int t = 0; t < n_act && ok; ++t) {  // t: position in the active list
        const int s = ((NPASS - 1) * n_act + t) % kQStagesK;
        const int db = t & 1;
        if (!(ok = mbar_wait(&bars->ds_full[db], (t >> 1) & 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bd = sw128_desc(k_base + s * TILE + kk * 16 * 128, kHalf, 1024);
          mma_f16_ts(tmem_dq, tmem_ds + db * 64 + kk * 8, bd, IDESC_DQ, t > 0 || kk > 0);
        }
        mma_commit(&bars->k_empty[s]);
        mma_commit(&bars->ds_empty[db]);
      }
      if (ok) mma_commit(&bars->dq_done);
      if (!ok) {
        *abort_ptr = 1;
        if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
      }
    }
  } else {
    // NWG warpgroups share each 128 x 128 tile: warpgroup wg owns key columns
    // [COLS wg, COLS (wg + 1)) of every row (TMEM lanes are reached through warp % 4).
    constexpr int NWG = Roles<HD>::NWG;
    constexpr int COLS = kBN / NWG;
    constexpr int CPW = COLS / 32;  // 32-column TMEM chunks per warpgroup
    const int wg = warp >> 2;
    const int row = threadIdx.x & 127;
    const int i = q0 + row;
    const bool row_ok = i < g.q_len;
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const int limit = i + g.shift;
    int vis_hi = row_ok ? g.k_len : 0;
    if (p.causal) vis_hi = min(vis_hi, limit + 1);
    int vis_lo = 0;
    if (p.window_left > 0) vis_lo = limit - p.window_left + 1;
    const float zs = zscale<NORM>(p.scale);
    float st0 = 0.f, inv_l = 1.f, c = 0.f;
    int64_t si = 0;
    if (row_ok) {
      si = stat_index(p, g, h, i);
      st0 = p.stats[si];
      inv_l = NORM == HFAN_SOFTMAX1 ? 1.f / p.stats[(int64_t)p.hq * p.rows_total + si] : 1.f;
    }
    // Sums (a, b) of this row over the warpgroups, through the dS TMEM
    // columns (idle until the first dS write; every thread touches only its
    // own lane, and the second barrier orders the reads before that write).
    auto row_exchange = [&](float a, float b, float* sa, float* sb) {
      tmem_st2(tmem_ds + lane_addr + 2 * wg, __float_as_uint(a), __float_as_uint(b));
      tmem_wait_st();
      tc_fence_before();
      named_bar_sync(1, Roles<HD>::ROW_THREADS);
      tc_fence_after();
      float ra = 0.f, rb = 0.f;
      if constexpr (NWG == 4) {
        uint32_t r[8];
        tmem_ld8(tmem_ds + lane_addr, r);
        tmem_wait_ld();
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
          ra += __uint_as_float(r[2 * w]);
          rb += __uint_as_float(r[2 * w + 1]);
        }
      } else {
        uint32_t r[4];
        tmem_ld4(tmem_ds + lane_addr, r);
        tmem_wait_ld();
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
          ra += __uint_as_float(r[2 * w]);
          rb += __uint_as_float(r[2 * w + 1]);
        }
      }
      tc_fence_before();
      named_bar_sync(1, Roles<HD>::ROW_THREADS);
      tc_fence_after();
      *sa = ra;
      *sb = rb;
    };
    if (NORM == HFAN_SOFTMAX1 || NPASS == 1) {
      // c = O . dO for softmax1 (the implicit sink carries no value) and
      // dO . wmean for the sparse normalizers (sum_j w_j dP_j / sum_j w_j with
      // dP_j = dO . v_j); warpgroup wg sums the head-dim slice
      // [HD/NWG wg, HD/NWG (wg + 1)), then the slices are combined.
      constexpr int DW = HD / NWG;
      float acc = 0.f;
      if (row_ok) {
        const T* orow = NORM == HFAN_SOFTMAX1
                            ? static_cast<const T*>(p.o) + qrow_off(p, g, b, h, i, p.o_sb, p.o_sh, p.o_st) + wg * DW
                            : static_cast<const T*>(p.wm) + qrow_off(p, g, b, h, i, p.wm_sb, p.wm_sh, p.wm_st) +
                                  wg * DW;
        const T* drow = static_cast<const T*>(p.dout) + qrow_off(p, g, b, h, i, p.do_sb, p.do_sh, p.do_st) + wg * DW;
#pragma unroll
        for (int d = 0; d < DW; d += 8) {
          uint4 ov = *reinterpret_cast<const uint4*>(orow + d);
          uint4 dv = *reinterpret_cast<const uint4*>(drow + d);
          const T* oe = reinterpret_cast<const T*>(&ov);
          const T* de = reinterpret_cast<const T*>(&dv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc = fmaf(to_f32<T>(oe[e]), to_f32<T>(de[e]), acc);
        }
      }
      float sum_unused;
      row_exchange(acc, 0.f, &c, &sum_unused);
    }
    bool ok = true;
    uint32_t sdc = 0;

    // Loads one 32-column chunk of S and dP as 16 packed pairs: x = s zs -
    // st0 (one packed FMA per pair; masked keys -> -inf, applied only on
    // tiles the mask cuts) and dP.
    const uint64_t zs2 = f2_pack(zs, zs), nst2 = f2_pack(-st0, -st0), il2 = f2_pack(inv_l, inv_l);
    // Dropout: the gradient reaching p is dP keep / (1 - p_drop) (same keep
    // bits as the forward, regenerated from the seed).
    constexpr bool drop = DROP;  // a separate instantiation: no cost without dropout
    uint32_t seed_lo = 0u, seed_hi = 0u;
    uint64_t drow = 0;
    if (drop) {
      const uint64_t sd = (uint64_t)*p.drop_seed;
      seed_lo = (uint32_t)sd;
      seed_hi = (uint32_t)(sd >> 32);
      drow = ((uint64_t)b * p.hq + h) * p.len_q + (row_ok ? i : 0);
    }
    auto chunk = [&](int t, int cidx, uint64_t (&x)[16], uint64_t (&dv)[16]) {
      uint32_t rs[32], rd[32];
      tmem_ld32(tmem_s + lane_addr + cidx * 32, rs);
      tmem_ld32(tmem_dp + lane_addr + cidx * 32, rd);
      tmem_wait_ld();
#pragma unroll
      for (int jp = 0; jp < 16; ++jp) {
        x[jp] = ffma2(f2_pack(__uint_as_float(rs[2 * jp]), __uint_as_float(rs[2 * jp + 1])), zs2, nst2);
        dv[jp] = f2_pack(__uint_as_float(rd[2 * jp]), __uint_as_float(rd[2 * jp + 1]));
      }
      const int kb = k_lo + t * kBN + cidx * 32;
      if (drop) {
#pragma unroll
        for (int g4 = 0; g4 < 8; ++g4) {
          const uint32_t keep = dropout_keep4(drow, (uint32_t)((kb >> 2) + g4), seed_lo, seed_hi, p.drop_thr24);
          const float k0 = (keep & 1u) ? p.drop_scale : 0.f, k1 = (keep & 2u) ? p.drop_scale : 0.f;
          const float k2 = (keep & 4u) ? p.drop_scale : 0.f, k3 = (keep & 8u) ? p.drop_scale : 0.f;
          dv[2 * g4] = fmul2(dv[2 * g4], f2_pack(k0, k1));
          dv[2 * g4 + 1] = fmul2(dv[2 * g4 + 1], f2_pack(k2, k3));
        }
      }
      const int lo = vis_lo - kb, hi = vis_hi - kb;
      if (!__all_sync(0xffffffffu, lo <= 0 && hi >= 32)) {
#pragma unroll
        for (int jp = 0; jp < 16; ++jp) {
          const int j = 2 * jp;
          x[jp] = f2_pack(j >= lo && j < hi ? f2_lo(x[jp]) : kNegInf,
                          j + 1 >= lo && j + 1 < hi ? f2_hi(x[jp]) : kNegInf);
        }
      }
    };
    // Weights of a pair (w = dp/dz up to the factor the normalizer's backward
    // folds in): softmax1 p = 2^x / l, sparsemax 1[x > 0], entmax15 (x)_+.
    auto wpair = [&](uint64_t x) -> uint64_t {
      if (NORM == HFAN_SOFTMAX1) return fmul2(f2_pack(ex2_ftz(f2_lo(x)), ex2_ftz(f2_hi(x))), il2);
      if (NORM == HFAN_SPARSEMAX) return f2_pack(f2_lo(x) > 0.f ? 1.f : 0.f, f2_hi(x) > 0.f ? 1.f : 0.f);
      return f2_pack(fmaxf(f2_lo(x), 0.f), fmaxf(f2_hi(x), 0.f));
    };

    if (SPARSE && NPASS == 2) {
      float num = 0.f, den = 0.f;
      for (int a = 0; a < n_act && ok; ++a) {
        const int t = tile_at(a);
        if (!(ok = wait_warp(&bars->sdp_full, sdc & 1, abort_flag))) break;
        tc_fence_after();
        uint64_t num2 = 0, den2 = 0;
#pragma unroll
        for (int cc = 0; cc < CPW; ++cc) {
          uint64_t x[16], dv[16];
          chunk(t, wg * CPW + cc, x, dv);
          if (cc == CPW - 1) {  // S and dP are in registers: the next tile's MMAs may overwrite them
            tc_fence_before();
            warp_arrive(&bars->sdp_empty);
          }
#pragma unroll
          for (int jp = 0; jp < 16; ++jp) {
            const uint64_t w = wpair(x[jp]);
            num2 = ffma2(w, dv[jp], num2);
            den2 = fadd2(den2, w);
          }
        }
        num += f2_lo(num2) + f2_hi(num2);
        den += f2_lo(den2) + f2_hi(den2);
        ++sdc;
      }
      // combine the warpgroups' column sums
      row_exchange(num, den, &num, &den);
      c = den > 0.f ? num / den : 0.f;
    }
    if (row_ok && wg == 0) p.corr[si] = c;

    for (int a = 0; a < n_act && ok; ++a) {
      const int t = tile_at(a);
      if (!(ok = wait_warp(&bars->sdp_full, sdc & 1, abort_flag))) break;
      tc_fence_after();
      uint32_t pk[COLS / 2];
      const uint64_t nc2 = f2_pack(-c, -c);
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) {
        uint64_t x[16], dv[16];
        chunk(t, wg * CPW + cc, x, dv);
        if (cc == CPW - 1) {  // S and dP are in registers: the next tile's MMAs may overwrite them
          tc_fence_before();
          warp_arrive(&bars->sdp_empty);
        }
#pragma unroll
        for (int jp = 0; jp < 16; ++jp) {
          // dS = w (dP - c)
          const uint64_t g2 = fadd2(dv[jp], nc2);
          uint64_t d2;
          if (NORM == HFAN_SPARSEMAX)
            d2 = f2_pack(f2_lo(x[jp]) > 0.f ? f2_lo(g2) : 0.f, f2_hi(x[jp]) > 0.f ? f2_hi(g2) : 0.f);
          else
            d2 = fmul2(wpair(x[jp]), g2);
          pk[cc * 16 + jp] = pack2<BF16>(f2_lo(d2), f2_hi(d2));
        }
      }
      ++sdc;
      // dS of list position a -> TMEM buffer a & 1, free once the dQ of
      // position a - 2 has completed
      const int db = a & 1;
      if (a >= 2) {
        if (!(ok = wait_warp(&bars->ds_empty[db], ((a >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
      }
#pragma unroll
      for (int cc = 0; cc < CPW; ++cc) tmem_st16(tmem_ds + lane_addr + db * 64 + wg * (COLS / 2) + cc * 16, pk + cc * 16);
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(&bars->ds_full[db]);
    }
    if (ok && n_act > 0) {
      ok = wait_warp(&bars->dq_done, 0, abort_flag);
      tc_fence_after();
    }
    if (!ok) {
      *abort_ptr = 1;
      if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
    }
    T* dqrow = static_cast<T*>(p.dq) + qrow_off(p, g, b, h, row_ok ? i : 0, p.dq_sb, p.dq_sh, p.dq_st);
#pragma unroll
    for (int cc = 0; cc < 1; ++cc) {
      const int cidx = wg;  // warpgroup wg stores head-dim columns [32 wg, 32 wg + 32)
      uint32_t r[32];
      if (n_act > 0) {
        tmem_ld32(tmem_dq + lane_addr + cidx * 32, r);
        tmem_wait_ld();
      }
      if (n_act == 0 || !ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(r[j + 0]) * p.scale, __uint_as_float(r[j + 1]) * p.scale);
          v.y = pack2<BF16>(__uint_as_float(r[j + 2]) * p.scale, __uint_as_float(r[j + 3]) * p.scale);
          v.z = pack2<BF16>(__uint_as_float(r[j + 4]) * p.scale, __uint_as_float(r[j + 5]) * p.scale);
          v.w = pack2<BF16>(__uint_as_float(r[j + 6]) * p.scale, __uint_as_float(r[j + 7]) * p.scale);
          *reinterpret_cast<uint4*>(dqrow + cidx * 32 + j) = v;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == Roles<HD>::MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =========================================================== dk/dv kernel
// One CTA per 128-key tile; units = (query head of the KV group, 64-row query
// tile).  Per unit: S^T = K Q^T and dP^T = V dO^T (M = 128 keys, N = 64
// queries) into one of two TMEM buffers, so that the next unit's products run
// while the row warps turn this unit's into P^T and dS^T; those go to two
// separate shared-memory tiles for dV += P^T dO and dK += dS^T Q (K = 64).
// Q / dO tiles (64 rows) stream through a 3-stage ring; the P^T / dS^T
// tiles are double-buffered, so that the row warps never wait for the
// previous unit's dV / dK.
constexpr int kQB = 64;        // query rows per unit
constexpr int kQStages = 3;    // Q / dO ring depth
constexpr uint32_t kQHalf = kQB * 128u;  // one 64-row x 128-byte swizzled half tile
constexpr int kUnitWords = 64;           // support bits of up to 2048 units per key tile

struct KBars {
  uint64_t kv_full;
  uint64_t qd_full[kQStages], qd_empty[kQStages];
  uint64_t sdp_full[2], sdp_empty[2], p_full[2], p_empty[2], done;
};

template <int HD>
struct KLayout {
  static constexpr int NH = HD / 64;
  static constexpr uint32_t K = 0;
  static constexpr uint32_t V = K + NH * kHalf;
  static constexpr uint32_t Q = V + NH * kHalf;                  // kQStages stages
  static constexpr uint32_t DO = Q + kQStages * NH * kQHalf;     // kQStages stages
  static constexpr uint32_t PP = DO + kQStages * NH * kQHalf;    // 2 x P^T  [128 keys][64 queries]
  static constexpr uint32_t PD = PP + 2 * kHalf;                 // 2 x dS^T [128 keys][64 queries]
  static constexpr uint32_t BARS = PD + 2 * kHalf;
  static constexpr uint32_t CTL = BARS + sizeof(KBars);
  static constexpr uint32_t MASK = CTL + 16;                   // [kUnitWords] units with support
  static constexpr uint32_t TOTAL = MASK + kUnitWords * 4 + 1024;
};

template <int HD, bool BF16, int NORM, bool DROP>
__global__ void __launch_bounds__(Roles<HD, 2>::THREADS, 1)
    tc_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const AttnParams p) {
  // the support lists are complete and every key segment was short enough:
  // sparse_list_bwd computed dK and dV
  if (NORM != HFAN_SOFTMAX1 && p.sl_flag != nullptr && *p.sl_flag == 0) return;
  using L = KLayout<HD>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int NH = L::NH;
  constexpr uint32_t TILE = NH * kHalf;     // K or V tile
  constexpr uint32_t QTILE = NH * kQHalf;   // Q or dO tile (64 rows)
  constexpr uint32_t IDESC_S = idesc_f16(BF16, kBN, kQB, false, false);
  constexpr uint32_t IDESC_ACC = idesc_f16(BF16, kBN, HD, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  KBars* bars = reinterpret_cast<KBars*>(smem + L::BARS);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::CTL);
  int* abort_ptr = reinterpret_cast<int*>(smem + L::CTL + 4);
  volatile int* abort_flag = abort_ptr;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint3 tile = tile_coords(p.tile_lpt);  // key tile 0 carries the most causal rows
  const int b = tile.z, kvh = tile.y;
  const Geometry g = geometry(p, b);
  const int k0 = tile.x * kBN;
  if (k0 >= g.k_len) return;
  const int groups = p.hq / p.hkv;
  const bool varlen = p.cu_q != nullptr;
  const int qtok0 = varlen ? g.q_start : 0;
  const int ktok = varlen ? g.k_start + k0 : k0;
  const int bcoord = varlen ? 0 : b;

  // query rows that see any key of this tile
  const int off = g.shift;
  int i_lo = 0;
  if (p.causal) i_lo = max(0, k0 - off);
  int i_hi = g.q_len;
  if (p.window_left > 0) i_hi = min(i_hi, min(k0 + kBN, g.k_len) - 1 - off + p.window_left);
  const int m_lo = i_lo / kQB;
  const int m_hi = i_hi > i_lo ? (i_hi + kQB - 1) / kQB : m_lo;
  const int n_m = m_hi - m_lo;
  const int n_units = groups * n_m;
  // Sparse normalizers skip the units whose probabilities against this key
  // tile are all zero (the forward's bit of (query head, 64-row block, tile)).
  uint32_t* ubits = reinterpret_cast<uint32_t*>(smem + L::MASK);
  const bool use_mask = NORM != HFAN_SOFTMAX1 && p.tile_mask != nullptr && n_units <= 32 * kUnitWords;
  if (use_mask) {
    const int kt = tile.x;
    for (int wi = warp; wi < (n_units + 31) / 32; wi += blockDim.x / 32) {
      const int u = wi * 32 + lane;
      bool bit = false;
      if (u < n_units) {
        const int hq = kvh * groups + u / n_m, m = m_lo + u % n_m;
        const uint32_t word =
            p.tile_mask[((int64_t)(hq * p.batch + b) * p.mask_qb + m) * p.mask_words + (kt >> 5)];
        bit = ((word >> (kt & 31)) & 1u) != 0u;
      }
      const unsigned bal = __ballot_sync(0xffffffffu, bit);
      if (lane == 0) ubits[wi] = bal;
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    for (int s = 0; s < kQStages; ++s) {
      mbar_init(&bars->qd_full[s], 1);
      mbar_init(&bars->qd_empty[s], 1);
    }
    // the S^T / dP^T buffer and the P^T / dS^T tiles of a list position are
    // consumed and produced by one row group (NGRP groups take turns)
    constexpr int GROUP_WARPS = Roles<HD>::ROW_THREADS / 32 / (Roles<HD>::NWG >= 4 ? 2 : 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->sdp_full[s], 1);
      mbar_init(&bars->sdp_empty[s], GROUP_WARPS);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->p_full[s], GROUP_WARPS);
      mbar_init(&bars->p_empty[s], 1);
    }
    mbar_init(&bars->done, 1);
    *abort_ptr = 0;
    fence_barrier_init();
  }
  if (warp == Roles<HD>::MMA_WARP) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM: S^T buffers [0, 64) and [64, 128), dP^T buffers [128, 192) and
  // [192, 256), dV [256, 256 + HD), dK [256 + HD, 256 + 2 HD)
  const uint32_t tmem_s = tmem, tmem_dp = tmem + 128, tmem_dv = tmem + 256, tmem_dk = tmem + 256 + HD;
  // Active units in increasing order; every role walks the same list, and
  // ring stages and buffer parities count list positions.
  const uint32_t* ubits_or_all = use_mask ? ubits : nullptr;
  const bool has_units = BitWalk(ubits_or_all, n_units).next() < n_units;
  // number of active units (the MMA issuers count list positions only)
  auto count_units = [&]() -> int {
    if (!use_mask) return n_units;
    int c = 0;
    for (int w = 0; w < (n_units + 31) / 32; ++w) c += __popc(ubits[w]);
    return c;
  };

  if (warp == Roles<HD>::TMA_WARP) {
    if (lane == 0 && has_units) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_do);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&bars->kv_full, 2 * TILE);
      for (int hh = 0; hh < NH; ++hh) {
        tma_load_4d(smem + L::K + hh * kHalf, &tm_k, &bars->kv_full, 64 * hh, ktok, kvh, bcoord);
        tma_load_4d(smem + L::V + hh * kHalf, &tm_v, &bars->kv_full, 64 * hh, ktok, kvh, bcoord);
      }
      bool ok = true;
      BitWalk walk(ubits_or_all, n_units);
      for (int a = 0, u = walk.next(); u < n_units && ok; ++a, u = walk.next()) {
        const int hq = kvh * groups + u / n_m;
        const int m = m_lo + u % n_m;
        const int s = a % kQStages;
        if (!(ok = mbar_wait(&bars->qd_empty[s], ((a / kQStages) & 1) ^ 1, abort_flag))) break;
        mbar_arrive_expect_tx(&bars->qd_full[s], 2 * QTILE);
        for (int hh = 0; hh < NH; ++hh) {
          tma_load_4d(smem + L::Q + s * QTILE + hh * kQHalf, &tm_q, &bars->qd_full[s], 64 * hh, qtok0 + m * kQB, hq,
                      bcoord);
          tma_load_4d(smem + L::DO + s * QTILE + hh * kQHalf, &tm_do, &bars->qd_full[s], 64 * hh, qtok0 + m * kQB,
                      hq, bcoord);
        }
      }
      if (!ok) {
        *abort_ptr = 1;
        if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
      }
    }
  } else if (warp == Roles<HD>::MMA_WARP) {
    // S^T and dP^T issuer
    if (lane == 0 && has_units) {
      const uint32_t k_base = smem_u32(smem + L::K), v_base = smem_u32(smem + L::V);
      const uint32_t q_base = smem_u32(smem + L::Q), do_base = smem_u32(smem + L::DO);
      bool ok = mbar_wait(&bars->kv_full, 0, abort_flag);
      const int n_act = count_units();
      for (int a = 0; a < n_act && ok; ++a) {
        const int s = a % kQStages, bf = a & 1;
        if (!(ok = mbar_wait(&bars->qd_full[s], (a / kQStages) & 1, abort_flag))) break;
        if (!(ok = mbar_wait(&bars->sdp_empty[bf], ((a >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t o = (kk >> 2) * kHalf + (kk & 3) * 32, oq = (kk >> 2) * kQHalf + (kk & 3) * 32;
          mma_f16_ss(tmem_s + bf * kQB, sw128_desc(k_base + o, 16, 1024), sw128_desc(q_base + s * QTILE + oq, 16, 1024),
                     IDESC_S, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t o = (kk >> 2) * kHalf + (kk & 3) * 32, oq = (kk >> 2) * kQHalf + (kk & 3) * 32;
          mma_f16_ss(tmem_dp + bf * kQB, sw128_desc(v_base + o, 16, 1024),
                     sw128_desc(do_base + s * QTILE + oq, 16, 1024), IDESC_S, kk > 0);
        }
        mma_commit(&bars->sdp_full[bf]);
      }
      if (!ok) {
        *abort_ptr = 1;
        if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
      }
    }
  } else if (warp == Roles<HD>::MMA2_WARP) {
    // dV += P^T dO and dK += dS^T Q per unit; then the P^T / dS^T tiles and
    // the unit's Q / dO stage are free (the unit's S^T / dP^T products
    // completed before P^T existed).
    if (lane == 0 && has_units) {
      const uint32_t q_base = smem_u32(smem + L::Q), do_base = smem_u32(smem + L::DO);
      const uint32_t pp_base = smem_u32(smem + L::PP), pd_base = smem_u32(smem + L::PD);
      bool ok = true;
      const int n_act = count_units();
      for (int a = 0; a < n_act && ok; ++a) {
        const int s = a % kQStages, pb = a & 1;
        if (!(ok = mbar_wait(&bars->p_full[pb], (a >> 1) & 1, abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kQB / 16; ++kk) {
          // A = P^T / dS^T [128 keys x 64 queries], K-major; B = dO / Q tile,
          // MN-major (rows = queries, 64-wide head-dim blocks kQHalf apart)
          const uint64_t bo = sw128_desc(do_base + s * QTILE + kk * 16 * 128, kQHalf, 1024);
          mma_f16_ss(tmem_dv, sw128_desc(pp_base + pb * kHalf + kk * 32, 16, 1024), bo, IDESC_ACC, a > 0 || kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < kQB / 16; ++kk) {
          const uint64_t bq = sw128_desc(q_base + s * QTILE + kk * 16 * 128, kQHalf, 1024);
          mma_f16_ss(tmem_dk, sw128_desc(pd_base + pb * kHalf + kk * 32, 16, 1024), bq, IDESC_ACC, a > 0 || kk > 0);
        }
        mma_commit(&bars->p_empty[pb]);
        mma_commit(&bars->qd_empty[s]);
      }
      if (ok) mma_commit(&bars->done);
      if (!ok) {
        *abort_ptr = 1;
        if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
      }
    }
  } else {
    // Row warps.  Thread = TMEM lane = key of the tile.  The row warpgroups
    // form NGRP independent groups that take the active units in turn (group
    // g: list positions a with a % NGRP == g), so one group's TMEM loads,
    // shared-memory stores and barrier waits overlap the other's arithmetic;
    // with two groups, group g always uses S^T / dP^T buffer g and P^T / dS^T
    // tile pair g.  A thread covers COLS = 32 query columns of its unit, in two
    // steps of 16.  The row statistics of those 32 queries sit one per lane and
    // are broadcast with shuffles (no shared-memory staging, no barrier
    // between the warps).
    constexpr int NWG = Roles<HD>::NWG;
    constexpr int NGRP = NWG >= 4 ? 2 : 1;  // independent row groups
    constexpr int GWG = NWG / NGRP;         // warpgroups per group
    constexpr int COLS = kQB / GWG;         // query columns per thread
    static_assert(COLS == 32, "one statistic per lane");
    const int wg = warp >> 2;
    const int grp = wg / GWG, sg = wg % GWG;
    const int cb = sg * COLS;           // this thread's first query column of a unit
    const int row = threadIdx.x & 127;  // key within the tile
    const int j = k0 + row;
    const bool key_ok = j < g.k_len;
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const float zs = zscale<NORM>(p.scale);
    constexpr bool drop = DROP;  // a separate instantiation: no cost without dropout
    uint32_t seed_lo = 0u, seed_hi = 0u;
    if (drop) {
      const uint64_t sd = (uint64_t)*p.drop_seed;
      seed_lo = (uint32_t)sd;
      seed_hi = (uint32_t)(sd >> 32);
    }
    bool ok = true;
    // Statistics of query column cb + lane of unit uu, negated where the
    // arithmetic subtracts them: -st0 (log2 max or tau), 1/l (softmax1) and -c.
    // Rows past the sequence read as st0 = +inf: x = -inf, p = 0.
    auto load_stats = [&](int uu, float& nst, float& il, float& nc) {
      nst = kNegInf;
      il = 1.f;
      nc = 0.f;
      if (uu >= n_units) return;
      const int iq = (m_lo + uu % n_m) * kQB + cb + lane;
      if (iq < g.q_len) {
        const int64_t si = stat_index(p, g, kvh * groups + uu / n_m, iq);
        nst = -p.stats[si];
        if (NORM == HFAN_SOFTMAX1) il = 1.f / p.stats[(int64_t)p.hq * p.rows_total + si];
        nc = -p.corr[si];
      }
    };
    // This group's units in list order, with their list positions.
    BitWalk walk(ubits_or_all, n_units);
    int a_walk = -1;
    auto next_mine = [&](int* pos) -> int {
      int uu;
      do {
        uu = walk.next();
        ++a_walk;
      } while (uu < n_units && a_walk % NGRP != grp);
      *pos = a_walk;
      return uu;
    };
    int a, a_n;
    int u = next_mine(&a), u_n = next_mine(&a_n);
    float nst_c, il_c, nc_c, nst_n, il_n, nc_n;
    load_stats(u, nst_c, il_c, nc_c);
    load_stats(u_n, nst_n, il_n, nc_n);
    while (u < n_units) {
      const int m = m_lo + u % n_m;
      const int qbase = m * kQB;
      const int bf = a & 1;
      if (!(ok = wait_warp(&bars->sdp_full[bf], (a >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      // visible queries of this key: [c_lo, c_hi) relative to qbase
      const int jl = j - off;  // causal: query i sees key j iff i >= j - off
      int c_lo = p.causal ? jl - qbase : -1 << 30;
      int c_hi = key_ok ? g.q_len - qbase : -(1 << 30);
      if (p.window_left > 0) c_hi = min(c_hi, jl + p.window_left - qbase);
      const int lo = c_lo - cb, hi = c_hi - cb;
      const bool full = __all_sync(0xffffffffu, lo <= 0 && hi >= COLS);
      const uint64_t zs2 = f2_pack(zs, zs);
      const int hqu = kvh * groups + u / n_m;
      uint32_t ppk[COLS / 2], dpk[COLS / 2];
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t rs[16], rd[16];
        tmem_ld16(tmem_s + bf * kQB + lane_addr + cb + 16 * hf, rs);
        tmem_ld16(tmem_dp + bf * kQB + lane_addr + cb + 16 * hf, rd);
        tmem_wait_ld();
        if (hf == 1) {
          tc_fence_before();
          warp_arrive(&bars->sdp_empty[bf]);  // the group's next unit may reuse this buffer
        }
#pragma unroll
        for (int e2 = 0; e2 < 16; e2 += 2) {
          const int e = 16 * hf + e2;  // column within the thread's 32
          const uint64_t nst = f2_pack(__shfl_sync(0xffffffffu, nst_c, e), __shfl_sync(0xffffffffu, nst_c, e + 1));
          const uint64_t nc2 = f2_pack(__shfl_sync(0xffffffffu, nc_c, e), __shfl_sync(0xffffffffu, nc_c, e + 1));
          uint64_t x = ffma2(f2_pack(__uint_as_float(rs[e2]), __uint_as_float(rs[e2 + 1])), zs2, nst);
          if (!full)
            x = f2_pack(e >= lo && e < hi ? f2_lo(x) : kNegInf, e + 1 >= lo && e + 1 < hi ? f2_hi(x) : kNegInf);
          uint64_t g2, ks2 = 0;
          if (drop) {  // keep / (1 - p_drop) of (query row, this key), as in the forward
            const uint64_t r0 = ((uint64_t)b * p.hq + hqu) * p.len_q + (qbase + cb + e);
            const uint32_t jg = (uint32_t)(j >> 2), js = (uint32_t)(j & 3);
            const uint32_t w0 = (dropout_keep4(r0, jg, seed_lo, seed_hi, p.drop_thr24) >> js) & 1u;
            const uint32_t w1 = (dropout_keep4(r0 + 1, jg, seed_lo, seed_hi, p.drop_thr24) >> js) & 1u;
            ks2 = f2_pack(w0 ? p.drop_scale : 0.f, w1 ? p.drop_scale : 0.f);
            g2 = ffma2(f2_pack(__uint_as_float(rd[e2]), __uint_as_float(rd[e2 + 1])), ks2, nc2);
          } else {
            g2 = fadd2(f2_pack(__uint_as_float(rd[e2]), __uint_as_float(rd[e2 + 1])), nc2);
          }
          uint64_t pr, ds;
          if (NORM == HFAN_SOFTMAX1) {
            const uint64_t il = f2_pack(__shfl_sync(0xffffffffu, il_c, e), __shfl_sync(0xffffffffu, il_c, e + 1));
            pr = fmul2(f2_pack(ex2_ftz(f2_lo(x)), ex2_ftz(f2_hi(x))), il);
            ds = fmul2(pr, g2);
          } else if (NORM == HFAN_SPARSEMAX) {
            pr = f2_pack(fmaxf(f2_lo(x), 0.f), fmaxf(f2_hi(x), 0.f));
            ds = f2_pack(f2_lo(x) > 0.f ? f2_lo(g2) : 0.f, f2_hi(x) > 0.f ? f2_hi(g2) : 0.f);
          } else {
            const uint64_t d = f2_pack(fmaxf(f2_lo(x), 0.f), fmaxf(f2_hi(x), 0.f));
            pr = fmul2(d, d);
            ds = fmul2(d, g2);
          }
          if (drop) pr = fmul2(pr, ks2);  // dV takes the dropped probabilities
          ppk[e / 2] = pack2<BF16>(f2_lo(pr), f2_hi(pr));
          dpk[e / 2] = pack2<BF16>(f2_lo(ds), f2_hi(ds));
        }
      }
      // P^T / dS^T tile pair a & 1 is free once the dV / dK of list position a - 2 completed
      const int pb = a & 1;
      if (a >= 2) {
        if (!(ok = wait_warp(&bars->p_empty[pb], ((a >> 1) & 1) ^ 1, abort_flag))) break;
      }
      store_chunks_sw128<COLS / 8>(smem + L::PP + pb * kHalf, row, cb / 8, ppk);
      store_chunks_sw128<COLS / 8>(smem + L::PD + pb * kHalf, row, cb / 8, dpk);
      fence_proxy_async_smem();
      tc_fence_before();
      warp_arrive(&bars->p_full[pb]);
      // the group's next unit (its statistics were loaded during this one)
      u = u_n;
      a = a_n;
      nst_c = nst_n;
      il_c = il_n;
      nc_c = nc_n;
      u_n = next_mine(&a_n);
      load_stats(u_n, nst_n, il_n, nc_n);
    }
    if (ok && has_units) {
      ok = wait_warp(&bars->done, 0, abort_flag);
      tc_fence_after();
    }
    if (!ok) {
      *abort_ptr = 1;
      if (p.dev_status) atomicCAS(p.dev_status, kDevOk, kDevWaitTimeout);
    }
    const int64_t kt = varlen ? (int64_t)g.k_start + (key_ok ? j : 0) : (key_ok ? j : 0);
    const int64_t boff = varlen ? 0 : (int64_t)b;
    T* dkrow = static_cast<T*>(p.dk) + boff * p.dk_sb + (int64_t)kvh * p.dk_sh + kt * p.dk_st;
    T* dvrow = static_cast<T*>(p.dv) + boff * p.dv_sb + (int64_t)kvh * p.dv_sh + kt * p.dv_st;
    // dV (columns 0..HD-1) then dK (HD..2HD-1): 2 HD / 32 chunks, two per warpgroup
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int chunk_id = wg * 2 + q;
      const int which = chunk_id / (HD / 32);
      const int cidx = chunk_id % (HD / 32);
      const uint32_t src = which == 0 ? tmem_dv : tmem_dk;
      const float f = which == 0 ? 1.f : p.scale;
      T* dst = which == 0 ? dvrow : dkrow;
      {
        uint32_t r[32];
        if (has_units) {
          tmem_ld32(src + lane_addr + cidx * 32, r);
          tmem_wait_ld();
        }
        if (!has_units || !ok) {
#pragma unroll
          for (int x = 0; x < 32; ++x) r[x] = 0u;
        }
        if (key_ok) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 v;
            v.x = pack2<BF16>(__uint_as_float(r[x + 0]) * f, __uint_as_float(r[x + 1]) * f);
            v.y = pack2<BF16>(__uint_as_float(r[x + 2]) * f, __uint_as_float(r[x + 3]) * f);
            v.z = pack2<BF16>(__uint_as_float(r[x + 4]) * f, __uint_as_float(r[x + 5]) * f);
            v.w = pack2<BF16>(__uint_as_float(r[x + 6]) * f, __uint_as_float(r[x + 7]) * f);
            *reinterpret_cast<uint4*>(dst + cidx * 32 + x) = v;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == Roles<HD>::MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// =========================================================== host
template <typename K>
cudaError_t launch_k(K kernel, dim3 grid, int threads, size_t smem, cudaStream_t s, const CUtensorMap& a,
                     const CUtensorMap& b, const CUtensorMap& c, const CUtensorMap& d, const AttnParams& p) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kernel<<<grid, threads, smem, s>>>(a, b, c, d, p);
  return cudaGetLastError();
}

template <int HD, bool BF16, int NORM>
cudaError_t launch_bwd_t(const AttnParams& p, int max_q, int max_k, cudaStream_t s) {
  const bool varlen = p.cu_q != nullptr;
  const int64_t tq = varlen ? p.rows_total : p.len_q;
  const int64_t tk = varlen ? p.rows_k : p.len_k;
  const int batch = varlen ? 1 : p.batch;
  CUtensorMap mq, mdo, mk, mv;
  if (!make_map(&mq, p.q, BF16, HD, tq, p.hq, batch, p.q_st, p.q_sh, varlen ? tq * p.q_st : p.q_sb) ||
      !make_map(&mdo, p.dout, BF16, HD, tq, p.hq, batch, p.do_st, p.do_sh, varlen ? tq * p.do_st : p.do_sb) ||
      !make_map(&mk, p.k, BF16, HD, tk, p.hkv, batch, p.k_st, p.k_sh, varlen ? tk * p.k_st : p.k_sb) ||
      !make_map(&mv, p.v, BF16, HD, tk, p.hkv, batch, p.v_st, p.v_sh, varlen ? tk * p.v_st : p.v_sb))
    return cudaErrorInvalidValue;
  // the dK/dV kernel streams 64-row Q / dO tiles
  CUtensorMap mq64, mdo64;
  if (!make_map(&mq64, p.q, BF16, HD, tq, p.hq, batch, p.q_st, p.q_sh, varlen ? tq * p.q_st : p.q_sb, kQB) ||
      !make_map(&mdo64, p.dout, BF16, HD, tq, p.hq, batch, p.do_st, p.do_sh, varlen ? tq * p.do_st : p.do_sb, kQB))
    return cudaErrorInvalidValue;
  AttnParams pq = p, pk = p;  // query tiles re-read K and V; key tiles re-read Q and dO
  pq.tile_lpt = (int64_t)batch * tk * p.hkv * HD * 4 <= kLptMaxReread;
  pk.tile_lpt = (int64_t)batch * tq * p.hq * HD * 4 <= kLptMaxReread;
  if (p.drop_thr24 != 0u) {
    cudaError_t e = launch_k(tc_bwd_dq_kernel<HD, BF16, NORM, true>, dim3((max_q + kBM - 1) / kBM, p.hq, p.batch),
                             Roles<HD, 2>::THREADS, QLayout<HD>::TOTAL, s, mq, mdo, mk, mv, pq);
    if (e != cudaSuccess) return e;
    return launch_k(tc_bwd_dkdv_kernel<HD, BF16, NORM, true>, dim3((max_k + kBN - 1) / kBN, p.hkv, p.batch),
                    Roles<HD, 2>::THREADS, KLayout<HD>::TOTAL, s, mq64, mdo64, mk, mv, pk);
  }
  cudaError_t e = cudaSuccess;
  // Support lists from the forward: the list kernels compute dQ, c, dK and
  // dV, and the tile kernels return at once (all read the overflow flags).
  if (NORM != HFAN_SOFTMAX1 && p.sl_ent != nullptr) e = sparse_list_bwd(BF16 ? HFAN_BFLOAT16 : HFAN_FLOAT16, p, s);
  if (e != cudaSuccess) return e;
  e = launch_k(tc_bwd_dq_kernel<HD, BF16, NORM, false>, dim3((max_q + kBM - 1) / kBM, p.hq, p.batch),
               Roles<HD, 2>::THREADS, QLayout<HD>::TOTAL, s, mq, mdo, mk, mv, pq);
  if (e != cudaSuccess) return e;
  return launch_k(tc_bwd_dkdv_kernel<HD, BF16, NORM, false>, dim3((max_k + kBN - 1) / kBN, p.hkv, p.batch),
                  Roles<HD, 2>::THREADS, KLayout<HD>::TOTAL, s, mq64, mdo64, mk, mv, pk);
}

template <int HD, bool BF16>
cudaError_t launch_bwd(const AttnParams& p, int max_q, int max_k, cudaStream_t s) {
  switch (p.norm) {
    case HFAN_SOFTMAX1: return launch_bwd_t<HD, BF16, HFAN_SOFTMAX1>(p, max_q, max_k, s);
    case HFAN_SPARSEMAX: return launch_bwd_t<HD, BF16, HFAN_SPARSEMAX>(p, max_q, max_k, s);
    default: return launch_bwd_t<HD, BF16, HFAN_ENTMAX15>(p, max_q, max_k, s);
  }
}

}  // namespace

cudaError_t tc_attention_bwd(int dtype, const AttnParams& p, int max_q, int max_k, cudaStream_t s) {
  // Gradients in the input dtype only; float32 gradient requests use the
  // general kernels.
  if (p.grad_f32) return cudaErrorNotSupported;
  if (!tc::aligned16(p.dout) || !tc::aligned16(p.dq) || !tc::aligned16(p.dk) || !tc::aligned16(p.dv) ||
      !tc::stride_ok(p.do_st) || !tc::stride_ok(p.do_sh) || (p.dq_st % 8) || (p.dq_sh % 8) ||
      (p.dk_st % 8) || (p.dk_sh % 8) || (p.dv_st % 8) || (p.dv_sh % 8))
    return cudaErrorNotSupported;
  if (p.cu_q == nullptr && p.batch > 1 &&
      (!tc::stride_ok(p.do_sb) || (p.dq_sb % 8) || (p.dk_sb % 8) || (p.dv_sb % 8)))
    return cudaErrorNotSupported;
  const bool bf16 = dtype == HFAN_BFLOAT16;
  if (p.d == 128) return bf16 ? launch_bwd<128, true>(p, max_q, max_k, s) : launch_bwd<128, false>(p, max_q, max_k, s);
  return bf16 ? launch_bwd<64, true>(p, max_q, max_k, s) : launch_bwd<64, false>(p, max_q, max_k, s);
}

}  // namespace hfan
