// Tensor-core fused attention forward for 16-bit inputs on sm_100a.
//
// One CTA computes 128 query rows of one (batch, query head) against all
// visible keys of its KV head, in key tiles of 128.  Warp roles (HD = head
// dim, NWG = HD / 32 row warpgroups: 4 at HD = 128, 2 at HD = 64):
//
//   warps 0 .. 4 NWG - 1   row warps: warpgroup wg owns key columns
//                          [128/NWG wg, 128/NWG (wg + 1)) of every S tile and
//                          head-dim columns [32 wg, 32 wg + 32) of O; thread =
//                          TMEM lane = query row.  They read S with tcgen05.ld,
//                          write P as packed 16-bit pairs into TMEM (the A
//                          operand of the P V MMA) and finalise O.
//   warp 4 NWG             TMA producer: Q once, then K and V tiles through one
//                          ring of 32 KB stages (5 at HD = 128, 8 at HD = 64)
//                          in the order the MMA warps consume them.
//   warp 4 NWG + 1         MMA issuer 1: S = Q K^T into a double-buffered TMEM tile.
//   warp 4 NWG + 2         MMA issuer 2: O += P V (TMEM accumulator).
//
// softmax1 runs one pass with an online max / denominator seeded with the
// implicit zero logit (m = 0, l = 1; reference kernels/softmax1_hopper.py:80-83);
// the O accumulator is rescaled lazily, only when a row max grows by more
// than 2^8.
//
// sparsemax / entmax15 need the row threshold tau before any probability is
// known, so they run a scan pass first (S only, no V).  Each row appends the
// scores above a rising lower bound of tau to a shared-memory candidate
// buffer (see Cand below); solving the threshold equation on that buffer gives
// the exact tau of vutils/entmax.py:35-133 without sorting.  Rows whose
// candidates outgrow the buffer continue with exact bracket sweeps over the
// whole row (common.cuh, tau_step).  The final pass then forms
// p = (z - tau)_+^a and P V; the output needs no normalisation.  It also
// records, per 64-row half and key tile, whether any p > 0 (p.tile_mask):
// the backward skips the tiles without support.  When every sparsemax row of
// the CTA has its whole support in the candidate buffers (key index beside
// each score), the final pass is skipped: P V and the w-weighted mean of V are gathered from the
// buffered support, which is also written out as the row's support list for
// the list backward (sparse_bwd.cu).  Optional dropout multiplies
// the P fed to P V by keep / (1 - p_drop) (Philox keep bits, common.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "params.cuh"
#include "tc_ptx.cuh"
#include "tc_common.cuh"

// Diagnostics (compiled in with -DHFAN_DIAG only): per-CTA clock64 sums of
// the scan / solve / final phases and counters of compactions and sweeps,
// read back with hfan_diag_read.  The product build contains none of it.
#ifdef HFAN_DIAG
__device__ unsigned long long g_hfan_diag[24];
extern "C" int hfan_diag_read(unsigned long long* out) {
  return (int)cudaMemcpyFromSymbol(out, g_hfan_diag, sizeof(unsigned long long) * 24);
}
extern "C" int hfan_diag_clear() {
  unsigned long long z[24] = {0};
  return (int)cudaMemcpyToSymbol(g_hfan_diag, z, sizeof(z));
}
#define DIAG_ADD(i, v) atomicAdd(&g_hfan_diag[i], (unsigned long long)(v))
#define DIAG_T(acc, stmt)               \
  do {                                  \
    const long long t0_ = clock64();    \
    stmt;                               \
    acc += clock64() - t0_;             \
  } while (0)
#else
#define DIAG_ADD(i, v) ((void)0)
#define DIAG_T(acc, stmt) stmt
#endif

namespace hfan {
namespace {

using namespace tc;

constexpr int kBM = 128;           // query rows per CTA
constexpr int kBN = 128;           // keys per tile
// K/V tiles share one ring of 128-row stages.  The scan and sweep passes
// (K only) cycle through the first kScanStages; the stages after them hold
// the candidate buffers meanwhile.  The final pass cycles through all of them,
// loading in the order the MMA warp consumes: K0 K1 V0 K2 V1 ... V(n-1).
template <int HD>
constexpr int ring_stages() { return HD == 128 ? 5 : 8; }
constexpr int kScanStages = 2;
#ifndef HFAN_CW
#define HFAN_CW 8
#endif
constexpr int kCW = HFAN_CW;                          // keys per chunk of the scan's gate
constexpr int kCompactRoom = kCW > 12 ? kCW : 12;     // free slots a compaction must leave
constexpr int kMaxStages = 8;
// The K-only passes (scan, sweeps) use all 512 TMEM columns as a 4-deep ring
// of S tiles (O, P and U are idle until the final pass), so row warps that
// run ahead or fall behind one another by up to three tiles do not hold up
// the next S = Q K^T.
constexpr int kKonlyBufs = 4;
constexpr int kMaxSweeps = 24;     // exact bracket sweeps before giving up
constexpr float kRescaleLog2 = 8.f;

// kPassGather: the sparse rows' supports are all in the candidate buffers, so
// the row warps gather P V from them and no final tensor-core pass runs.
enum Pass : int { kPassFinal = 0, kPassTopC = 1, kPassSweep = 2, kPassGather = 3 };

struct Bars {
  uint64_t q_full;
  uint64_t full[kMaxStages], empty[kMaxStages];
  uint64_t s_full[2], s_empty[2];
  uint64_t k_full[kKonlyBufs], k_empty[kKonlyBufs];  // S ring of the K-only passes
  uint64_t p_full[2], pv_done[2], ctrl;
};

struct Ctl {
  uint32_t tmem_base;
  int abort;
  int next_pass;
  int any_pending;
};

template <int HD>
struct Layout {
  static constexpr int NH = HD / 64;
  static constexpr uint32_t Q = 0;
  static constexpr int NS = ring_stages<HD>();
  static constexpr uint32_t RING = Q + NH * kHalf;
  static constexpr uint32_t CAND = RING + kScanStages * NH * kHalf;  // candidate buffers (scan/sweeps)
  static constexpr uint32_t CAND_BYTES = (NS - kScanStages) * NH * kHalf;
  static constexpr uint32_t BARS = RING + NS * NH * kHalf;
  static constexpr uint32_t CTL = BARS + sizeof(Bars);
  static constexpr uint32_t XCH_FLOATS = 6144 + 4 * 128;             // warpgroup exchange
  static constexpr uint32_t XCH = (CTL + sizeof(Ctl) + 15) & ~15u;
  static constexpr uint32_t MASK = XCH + XCH_FLOATS * 4;               // [2 row halves][kMaskWordsMax] key-tile bits
  static constexpr uint32_t TOTAL = MASK + 2 * kMaskWordsMax * 4 + 1024;  // + alignment slack
};

__device__ __forceinline__ void record_error(const AttnParams& p, Ctl* ctl, int code) {
  ctl->abort = 1;
  if (p.dev_status) atomicCAS(p.dev_status, kDevOk, code);
}

// ------------------------------------------------------------------ candidates
// Scan-pass state of one row.  Scores above the admission threshold `thr`
// (z units) are appended, unsorted, to the row's column of a shared-memory
// buffer buf[cap][128].  thr only rises and is always a lower bound of tau:
// it starts at (running max - 1) and is lifted to the exact threshold of the
// buffered candidates alone, whose f_A(t) = sum_A (z - t)_+^a never exceeds
// the row's f(t).  Every score above the final thr is therefore in the
// buffer, and the threshold solved on the buffer is the row's exact tau.
struct Cand {
  int n;          // buffered entries (some may be <= thr: dead, ignored)
  bool overflow;  // more live candidates than the buffer holds
  float thr;      // admission threshold, z units
  float thr_s;    // the same threshold in raw-score units (thr / zs, or slightly below it)
};

// A raw-score gate at or a few ulps below z / zs (izs = 1 / zs): a gate that
// is too low only admits a few dead entries, one that is too high could drop
// a candidate.  One multiply instead of a division on the scan's hot path.
__device__ __forceinline__ float raw_gate(float z, float izs) {
  const float r = z * izs;
  return r - fabsf(r) * 0x1p-20f;
}

// Solve f_A(t) = 1 on the buffered candidates starting from the lower bound
// t0 (exact bracket + closed form of common.cuh).  Returns the root (or the
// best lower bound after `max_iter` steps) and its support size.
template <int NORM>
__device__ float buffer_solve(const float* buf, int row, int n, float t0, int max_iter, bool* exact,
                              float* support) {
  float t = t0, tau = t0;
  *exact = false;
  for (int it = 0; it < max_iter; ++it) {
    TauStats st{0.f, 0.f, 0.f, kPosInf};
    for (int e = 0; e < n; ++e) tau_accumulate(st, buf[e * 128 + row], t);
    *support = st.cnt;
    if (st.cnt == 0.f) break;
    if (tau_step(NORM, st, &t, &tau)) {
      *exact = true;
      return tau;
    }
  }
  return t;
}

// Lower bound of tau from the KT largest chunk maxima zz[0] >= ... >= zz[KT-1]
// (z units, -inf when missing): any k distinct scores whose closed-form
// threshold t_k lies at or below the smallest of them give f(t_k) >= 1,
// hence t_k <= tau.  k = 1 is the zmax - 1 bound.
template <int NORM, int KT>
__device__ __forceinline__ float top_bound(const float (&zz)[KT]) {
  // The sizes k whose closed-form threshold t_k stays at or below the k-th
  // value form a prefix, and the largest one gives the set's threshold; the
  // test needs no root or division (1/k is a constant of the unrolled loop),
  // so a single closed form is evaluated at the end.
  const float z1 = zz[0];
  float s1 = 0.f, s2 = 0.f;
  float bt = 0.f, bmean = 0.f, bd = 0.f;  // the largest valid k's closed form (sparsemax) or its parts
  bool any = false;
#pragma unroll
  for (int k = 1; k <= KT; ++k) {
    const float y = zz[k - 1] - z1;
    s1 += y;
    s2 += y * y;
    const float inv = 1.f / float(k);
    bool valid;
    float tk = 0.f, mean = 0.f, d = 0.f;
    if (NORM == HFAN_SPARSEMAX) {
      tk = (s1 - 1.f) * inv;
      valid = tk <= y;
    } else {
      mean = s1 * inv;
      d = (1.f - (s2 - s1 * mean)) * inv;  // t_k = mean - sqrt(d)
      const float g = mean - y;             // t_k <= y  <=>  g <= sqrt(d)
      valid = g <= 0.f || (d >= 0.f && g * g <= d);
    }
    valid = valid && zz[k - 1] > kNegInf;
    if (valid) {
      any = true;
      bt = tk;
      bmean = mean;
      bd = d;
    }
  }
  if (!any) return z1 - 1.f;
  const float t = NORM == HFAN_SPARSEMAX ? bt : bmean - sqrtf(fmaxf(bd, 0.f));
  return fmaxf(z1 - 1.f, z1 + t);
}

// a >= b after the call
__device__ __forceinline__ void cswap(float& a, float& b) {
  const float hi = fmaxf(a, b);
  b = fminf(a, b);
  a = hi;
}

// t[0..3] (descending) becomes the four largest of t and the unsorted c[0..3]:
// c is sorted by a five-comparator network, the two sorted lists are folded
// into the bitonic top four (max of t[i] and c[3 - i]), and two compare
// levels sort it.  Depth 6 instead of the 16 of one insertion after another.
__device__ __forceinline__ void top4_merge(float (&t)[4], const float (&c)[4]) {
  float a = c[0], b = c[1], x = c[2], y = c[3];
  cswap(a, b);
  cswap(x, y);
  cswap(a, x);
  cswap(b, y);
  cswap(b, x);  // a >= b >= x >= y
  float r0 = fmaxf(t[0], y), r1 = fmaxf(t[1], x), r2 = fmaxf(t[2], b), r3 = fmaxf(t[3], a);
  cswap(r0, r2);
  cswap(r1, r3);
  cswap(r0, r1);
  cswap(r2, r3);
  t[0] = r0;
  t[1] = r1;
  t[2] = r2;
  t[3] = r3;
}

// The same solve over the NW per-warpgroup buffers of one row (buffer w holds
// ns[w] entries starting at entry w * capw).
template <int NORM, int NW>
__device__ float buffer_solve_multi(const float* buf0, int capw, int row, const int (&ns)[NW], float t0,
                                    int max_iter, bool* exact, float* support) {
  float t = t0, tau = t0;
  *exact = false;
  for (int it = 0; it < max_iter; ++it) {
    TauStats st{0.f, 0.f, 0.f, kPosInf};
#pragma unroll
    for (int w = 0; w < NW; ++w)
      for (int e = 0; e < ns[w]; ++e) tau_accumulate(st, buf0[(w * capw + e) * 128 + row], t);
    *support = st.cnt;
    if (st.cnt == 0.f) break;
    if (tau_step(NORM, st, &t, &tau)) {
      *exact = true;
      return tau;
    }
  }
  return t;
}

// Raise thr to the buffer's own threshold and drop dead entries.  State is
// passed by value so that callers keep it in registers.
template <int NORM, bool IDX>
__device__ __noinline__ Cand buffer_compact(float* buf, uint16_t* ibuf, int row, Cand c, int cap, float zs) {
  DIAG_ADD(0, 1);
  bool exact;
  float sup;
  float root = buffer_solve<NORM>(buf, row, c.n, c.thr, 8, &exact, &sup);
  if (root > c.thr) {
    c.thr = root;
    c.thr_s = root / zs;
  }
  int live = 0;
  for (int e = 0; e < c.n; ++e) {
    float z = buf[e * 128 + row];
    if (z > c.thr) {
      if (IDX) ibuf[live * 128 + row] = ibuf[e * 128 + row];
      buf[live++ * 128 + row] = z;
    }
  }
  c.n = live;
  // Stop buffering once compaction no longer frees room for a chunk of
  // appends.  Sparsemax (no cooperative vote) also stops when half the
  // buffer stays live: the row's candidates are dense, and compacting on
  // every chunk would cost more than the sweeps that settle such rows.
  if (live > (NORM == HFAN_SPARSEMAX ? cap / 2 : cap - kCompactRoom)) c.overflow = true;
  return c;
}

// Two 16-bit values (low half first in memory) -> packed f32x2.
template <bool BF16>
__device__ __forceinline__ uint64_t unpack2(uint32_t x) {
  if (BF16) return f2_pack(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&x));
  return f2_pack(f.x, f.y);
}

// ------------------------------------------------------------------ kernel
template <int HD, bool BF16, int NORM, bool DROP>
__global__ void __launch_bounds__(Roles<HD, 2>::THREADS, 1)
    tc_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const AttnParams p) {
  using L = Layout<HD>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int NH = L::NH;
  constexpr uint32_t KV_BYTES = NH * kHalf;
  constexpr uint32_t IDESC_QK = idesc_f16(BF16, kBM, kBN, false, false);
  constexpr uint32_t IDESC_PV = idesc_f16(BF16, kBM, HD, false, true);
  constexpr bool SPARSE = NORM != HFAN_SOFTMAX1;
#ifndef HFAN_KT_ENT
#define HFAN_KT_ENT 4
#endif
#ifndef HFAN_KT_SPM
#define HFAN_KT_SPM 4
#endif
#ifndef HFAN_VOTE_ITERS
#define HFAN_VOTE_ITERS 3
#endif
#ifndef HFAN_VOTE_MARGIN
#define HFAN_VOTE_MARGIN 20
#endif
#ifndef HFAN_VOTE_PERIOD
#define HFAN_VOTE_PERIOD 4
#endif
  constexpr bool SCAN = SPARSE;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + L::BARS);
  Ctl* ctl = reinterpret_cast<Ctl*>(smem + L::CTL);
  // Key tiles with any p > 0, per 64-row half of the tile (sparse final pass):
  // set by the row warps and written to p.tile_mask for the backward.
  uint32_t* sbits = reinterpret_cast<uint32_t*>(smem + L::MASK);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint3 tile = tile_coords(p.tile_lpt);
  const int b = tile.z, h = tile.y;
  const int qt = gridDim.x - 1 - tile.x;  // longest causal rows first
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
  const int kt0 = k_lo / kBN;  // absolute index of the first key tile
  // the support bits of every key tile fit in shared memory (and are wanted)
  const bool track = SPARSE && p.tile_mask != nullptr && kt0 + n_tiles <= 32 * kMaskWordsMax;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < L::NS; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_empty[s], Roles<HD>::ROW_THREADS / 32);
    }
    for (int s = 0; s < kKonlyBufs; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], Roles<HD>::ROW_THREADS / 32);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->p_full[s], Roles<HD>::ROW_THREADS / 32);
      mbar_init(&bars->pv_done[s], 1);
    }
    mbar_init(&bars->ctrl, 1);
    ctl->abort = 0;
    ctl->next_pass = kPassFinal;
    ctl->any_pending = 0;
    for (int w = 0; w < 2 * kMaskWordsMax; ++w) sbits[w] = 0u;
    fence_barrier_init();
  }
  if (warp == Roles<HD>::MMA_WARP) tmem_alloc(&ctl->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  const uint32_t tmem_o = tmem + 256;  // O: HD columns
  // P double buffer: 2 x 64 columns of packed 16-bit pairs.  Sparse with wmean
  // requested: [384, 384 + HD) accumulates U = sum_j w_j v_j instead, and P
  // and W (packed) overwrite each warpgroup's own columns of the S buffer they
  // came from (so S(t + 2) waits for P V(t) and W V(t)).
  const uint32_t tmem_p = tmem + 384;
  const uint32_t tmem_u = tmem + 384;
  const bool want_u = SPARSE && p.wm != nullptr;
  // per-row support lists for the sparse backward (no dropout)
  const bool lists = SPARSE && !DROP && p.sl_ent != nullptr;
  constexpr int PCOLS = kBN / Roles<HD>::NWG;  // keys per warpgroup and S tile
  volatile int* abort_flag = &ctl->abort;

  if (warp == Roles<HD>::TMA_WARP) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n_tiles > 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, NH * kHalf);
      for (int hh = 0; hh < NH; ++hh)
        tma_load_4d(smem + L::Q + hh * kHalf, &tm_q, &bars->q_full, 64 * hh, qtok, h, bcoord);
      // per-stage phase bits: a stage's empty barrier completes once per use
      uint32_t empty_ph = 0, ctrl_phase = 0;
      int ring = 0, ns = kScanStages;
      auto produce = [&](const CUtensorMap* map, int t) -> bool {
        const int st = ring;
        ring = ring + 1 == ns ? 0 : ring + 1;
        if (!mbar_wait(&bars->empty[st], ((empty_ph >> st) & 1) ^ 1, abort_flag)) return false;
        empty_ph ^= 1u << st;
        mbar_arrive_expect_tx(&bars->full[st], KV_BYTES);
        for (int hh = 0; hh < NH; ++hh)
          tma_load_4d(smem + L::RING + st * KV_BYTES + hh * kHalf, map, &bars->full[st], 64 * hh,
                      ktok0 + k_lo + t * kBN, kvh, bcoord);
        return true;
      };
      int pass = SCAN ? kPassTopC : kPassFinal;
      bool ok = true;
      while (ok) {
        const bool fin = pass == kPassFinal;
        ring = 0;
        ns = fin ? L::NS : kScanStages;
        for (int t = 0; t < n_tiles && ok; ++t) {
          ok = produce(&tm_k, t);
          if (ok && fin && t >= 1) ok = produce(&tm_v, t - 1);
        }
        if (ok && fin && n_tiles > 0) ok = produce(&tm_v, n_tiles - 1);
        if (!ok || fin) break;
        if (!(ok = mbar_wait(&bars->ctrl, ctrl_phase, abort_flag))) break;
        ctrl_phase ^= 1;
        pass = ctl->next_pass;
        if (pass == kPassGather) break;
      }
      if (!ok) record_error(p, ctl, kDevWaitTimeout);
    }
  } else if (warp == Roles<HD>::MMA_WARP || warp == Roles<HD>::MMA2_WARP) {
    // ------------------------------------------------------------ MMA issuers
    // tcgen05.mma issue is nearly synchronous with its execution, so every
    // wait of a single issuing thread would leave the tensor pipe idle.  Two
    // issuers: this warp's lane 0 issues S = Q K^T (every pass), the second
    // issuer's lane 0 issues O += P V (final pass); each one's barrier waits
    // overlap the other's MMAs.
    //
    // Ring bookkeeping shared by both: a K-only pass consumes items t = 0..n-1
    // from stages t % kScanStages; the final pass consumes K(t) as item
    // (t ? 2t - 1 : 0) and V(j) as item min(2j + 2, 2n - 1) from stages
    // item % NS.  A stage's full barrier has completed once per earlier use,
    // so the parity to wait for is (earlier uses) & 1.
    const bool qk_issuer = warp == Roles<HD>::MMA_WARP;
    if (lane == 0 && n_tiles > 0) {
      const uint32_t q_base = smem_u32(smem + L::Q);
      const uint32_t ring_base = smem_u32(smem + L::RING);
      // parity of the uses of each scan stage by the finished K-only passes
      uint32_t base_par = 0, ctrl_phase = 0;
      auto wait_item = [&](int idx, int nst, int* st) -> bool {
        const int s_ = idx % nst;
        const uint32_t par = ((uint32_t)(idx / nst) & 1u) ^ (s_ < kScanStages ? (base_par >> s_) & 1u : 0u);
        *st = s_;
        return mbar_wait(&bars->full[s_], par, abort_flag);
      };
      int pass = SCAN ? kPassTopC : kPassFinal;
      bool ok = qk_issuer ? mbar_wait(&bars->q_full, 0, abort_flag) : true;
      uint32_t sc = 0, kc = 0;  // S tiles issued in the final pass / in the K-only passes
      while (ok) {
        const bool fin = pass == kPassFinal;
        if (qk_issuer) {
          for (int t = 0; t < n_tiles && ok; ++t) {
            int ks;
            const int sb = fin ? (int)(sc & 1) : (int)(kc % kKonlyBufs);
            if (!(ok = wait_item(fin ? (t ? 2 * t - 1 : 0) : t, fin ? L::NS : kScanStages, &ks))) break;
            if (!fin) {
              if (!(ok = mbar_wait(&bars->k_empty[sb], ((kc / kKonlyBufs) & 1) ^ 1, abort_flag))) break;
            } else if (want_u && t >= 2) {
              // the buffer holds P and W of final-pass tile t - 2 until its P V is done
              if (!(ok = mbar_wait(&bars->pv_done[sb], ((t >> 1) & 1) ^ 1, abort_flag))) break;
            } else {
              if (!(ok = mbar_wait(&bars->s_empty[sb], ((sc >> 1) & 1) ^ 1, abort_flag))) break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint64_t a = sw128_desc(q_base + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = sw128_desc(ring_base + ks * KV_BYTES + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
              mma_f16_ss(tmem + sb * 128, a, bd, IDESC_QK, kk > 0);
            }
            mma_commit(fin ? &bars->s_full[sb] : &bars->k_full[sb]);
            mma_commit(&bars->empty[ks]);
            if (fin) ++sc; else ++kc;
          }
        } else if (fin) {
          // S buffer of final-pass tile j: j & 1 (the K-only passes have their own ring)
          for (int j = 0; j < n_tiles && ok; ++j) {
            int vs;
            const int pb = j & 1;
            if (!(ok = wait_item(min(2 * j + 2, 2 * n_tiles - 1), L::NS, &vs))) break;
            if (!(ok = mbar_wait(&bars->p_full[pb], (j >> 1) & 1, abort_flag))) break;
            tc_fence_after();
            if (want_u) {
              // A = P (and W) in the S buffer: keys [16 kk, 16 kk + 16) belong to
              // warpgroup 16 kk / PCOLS, whose P occupies the first PCOLS / 2
              // columns of its slice and W the next PCOLS / 2.
              const int sbj = j & 1;
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk) {
                const int wk = (16 * kk) / PCOLS, ko = 16 * kk - wk * PCOLS;
                const uint32_t pcol = (uint32_t)(sbj * 128 + wk * PCOLS + ko / 2);
                const uint64_t bd = sw128_desc(ring_base + vs * KV_BYTES + kk * 16 * 128, kHalf, 1024);
                mma_f16_ts(tmem_o, tmem + pcol, bd, IDESC_PV, j > 0 || kk > 0);
              }
              {
#pragma unroll
                for (int kk = 0; kk < kBN / 16; ++kk) {
                  const int wk = (16 * kk) / PCOLS, ko = 16 * kk - wk * PCOLS;
                  const uint32_t wcol = (uint32_t)(sbj * 128 + wk * PCOLS + PCOLS / 2 + ko / 2);
                  const uint64_t bd = sw128_desc(ring_base + vs * KV_BYTES + kk * 16 * 128, kHalf, 1024);
                  mma_f16_ts(tmem_u, tmem + wcol, bd, IDESC_PV, j > 0 || kk > 0);
                }
              }
              mma_commit(&bars->empty[vs]);
              mma_commit(&bars->pv_done[sbj]);
            } else {
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk) {
                // A = P [128 x 128 keys] in TMEM buffer pb (8 columns per 16 keys);
                // B = V tile, MN-major (rows = keys, 64-wide head-dim blocks kHalf apart).
                const uint64_t bd = sw128_desc(ring_base + vs * KV_BYTES + kk * 16 * 128, kHalf, 1024);
                mma_f16_ts(tmem_o, tmem_p + pb * 64 + kk * 8, bd, IDESC_PV, j > 0 || kk > 0);
              }
              mma_commit(&bars->empty[vs]);
              mma_commit(&bars->pv_done[pb]);
            }
          }
        }
        if (!ok || fin) break;
#pragma unroll
        for (int s_ = 0; s_ < kScanStages; ++s_) {
          const int uses = n_tiles > s_ ? (n_tiles - s_ + kScanStages - 1) / kScanStages : 0;
          base_par ^= (uint32_t)(uses & 1) << s_;
        }
        if (!(ok = mbar_wait(&bars->ctrl, ctrl_phase, abort_flag))) break;
        ctrl_phase ^= 1;
        pass = ctl->next_pass;
        if (pass == kPassGather) break;
      }
      if (!ok) record_error(p, ctl, kDevWaitTimeout);
    }
  } else if (warp < Roles<HD>::TMA_WARP) {
    // ------------------------------------------------------------ normalizer
    // NWG warpgroups share each 128-row tile: warpgroup wg owns key columns
    // [COLS wg, COLS (wg + 1)) of every S tile and head-dim columns
    // [32 wg, 32 wg + 32) of O.  Row-wide quantities (softmax1 max and
    // denominator, the sparse threshold) are combined through shared memory.
    constexpr int NWG = Roles<HD>::NWG;
    constexpr int NT = Roles<HD>::ROW_THREADS;
    constexpr int COLS = kBN / NWG;
    const int wg = warp >> 2;
    const int row = threadIdx.x & 127;  // TMEM lane
    const int i = q0 + row;             // query row within the sequence
    const bool row_ok = i < g.q_len;
    const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
    const int limit = i + g.shift;
    // visible keys of this row: [vis_lo, vis_hi)
    int vis_hi = row_ok ? g.k_len : 0;
    if (p.causal) vis_hi = min(vis_hi, limit + 1);
    int vis_lo = 0;
    if (p.window_left > 0) vis_lo = limit - p.window_left + 1;
    const float zs = NORM == HFAN_SOFTMAX1 ? p.scale * kLog2e
                                           : (NORM == HFAN_SPARSEMAX ? p.scale : 0.5f * p.scale);
    const float izs = 1.f / zs;
    // During the scan passes the V ring and the P buffer are idle; they hold
    // the candidate buffers (the producer loads V only in the final pass),
    // one slice per warpgroup.
    // Each entry: the score (z units, float) and, for sparsemax, its key
    // (uint16: the tile relative to k_lo above JB bits, the column in the
    // warpgroup's slice below), which the gather pass reads.  entmax15 keeps
    // the larger score-only buffers: its wider supports overflow the smaller
    // ones into whole-row sweeps.
    constexpr bool IDX = NORM == HFAN_SPARSEMAX;
    constexpr int CAPW = (int)(L::CAND_BYTES / (128 * (IDX ? 6 : 4))) / NWG;
    constexpr int JB = COLS == 32 ? 5 : 6;
    float* cbuf0 = reinterpret_cast<float*>(smem + L::CAND);
    float* cbuf = cbuf0 + wg * CAPW * 128;
    uint16_t* ibuf0 = reinterpret_cast<uint16_t*>(smem + L::CAND + NWG * CAPW * 128 * 4);
    uint16_t* ibuf = ibuf0 + wg * CAPW * 128;
    float* xch = reinterpret_cast<float*>(smem + L::XCH);  // [4096] floats

    uint32_t sc = 0, kc = 0, pc = 0;  // final-pass S tiles, K-only S tiles, P tiles
    bool ok = true;
    float sreg[COLS];  // raw scores s = q.k of this warpgroup's columns (masked: -inf)
#ifdef HFAN_DIAG
    long long dls_w = 0, dls_l = 0;
#endif
    // konly: an S tile of a K-only pass (4-deep ring, buffer kc % 4)
    auto load_s = [&](int t, bool konly) -> bool {
      const int sb = konly ? (int)(kc % kKonlyBufs) : (int)(sc & 1);
      uint64_t* sfull = konly ? &bars->k_full[sb] : &bars->s_full[sb];
      uint64_t* sempty = konly ? &bars->k_empty[sb] : &bars->s_empty[sb];
      const uint32_t sph = konly ? (kc / kKonlyBufs) & 1 : (sc >> 1) & 1;
#ifdef HFAN_DIAG
      long long c0_ = clock64();
#endif
      if (!wait_warp(sfull, sph, abort_flag)) return false;
      tc_fence_after();
#ifdef HFAN_DIAG
      long long c1_ = clock64();
      dls_w += c1_ - c0_;
#endif
      uint32_t r[COLS / 32][32];
#pragma unroll
      for (int c = 0; c < COLS / 32; ++c) tmem_ld32(tmem + lane_addr + sb * 128 + wg * COLS + c * 32, r[c]);
      tmem_wait_ld();
#ifdef HFAN_DIAG
      dls_l += clock64() - c1_;
#endif
      tc_fence_before();
      warp_arrive(sempty);
      if (konly) ++kc; else ++sc;
      const int kb = k_lo + t * kBN + wg * COLS;
      const int lo = vis_lo - kb, hi = vis_hi - kb;
      if (__all_sync(0xffffffffu, lo <= 0 && hi >= COLS)) {
#pragma unroll
        for (int j = 0; j < COLS; ++j) sreg[j] = __uint_as_float(r[j >> 5][j & 31]);
      } else {
#pragma unroll
        for (int j = 0; j < COLS; ++j) sreg[j] = (j >= lo && j < hi) ? __uint_as_float(r[j >> 5][j & 31]) : kNegInf;
      }
      return true;
    };

    // ---- threshold (sparse normalizers)
    float tau = kPosInf, support = 0.f;
    // Threshold of the union of this row's candidate buffers, starting from
    // the lower bound t0: every warpgroup sums its own buffer, the sums are
    // exchanged (double-buffered by iteration parity) and all warpgroups take
    // the same step; bar.red.or both synchronises and tells whether any row is
    // still iterating.  Every row thread must call it.  Returns true with the
    // exact root of the union in *out, or false with a lower bound of it.
    // With around_max the sums are taken around zref (the row maximum, the
    // same in every run), so that the exact root depends only on the support
    // and the fixed summation order (buffer order within a warpgroup, then
    // warpgroup order), not on the lower bound the search started from.
    auto union_solve = [&](const Cand& cdr, float t0, bool active, int max_iter, float* out, float* sup,
                           bool around_max = false, float zref = 0.f) -> bool {
      bool done = !active, exact = false;
      float tsol = t0;
      for (int it = 0;; ++it) {
        TauStats st{0.f, 0.f, 0.f, kPosInf};
        const float rr = around_max ? zref : tsol;
        if (!done)
          for (int e = 0; e < cdr.n; ++e) tau_accumulate_ref(st, cbuf[e * 128 + row], tsol, rr);
        float* xi = xch + 2048 + (it & 1) * (NWG * 512);  // [2][NWG][128][4]
        xi[(wg * 128 + row) * 4 + 0] = st.cnt;
        xi[(wg * 128 + row) * 4 + 1] = st.s1;
        xi[(wg * 128 + row) * 4 + 2] = st.s2;
        xi[(wg * 128 + row) * 4 + 3] = st.zmin;
        if (!named_bar_or(1, NT, !done)) break;
        if (done) continue;
        TauStats all{0.f, 0.f, 0.f, kPosInf};
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
          const float* o = xi + (w * 128 + row) * 4;
          all.cnt += o[0];
          all.s1 += o[1];
          all.s2 += o[2];
          all.zmin = fminf(all.zmin, o[3]);
        }
        *sup = all.cnt;
        float r;
        if (all.cnt == 0.f || it >= max_iter - 1) {
          done = true;
        } else if (tau_step_ref(NORM, all, rr, &tsol, &r)) {
          done = true;
          exact = true;
          tsol = r;
        }
      }
      *out = tsol;
      return exact;
    };
#ifdef HFAN_DIAG
    long long diag_t0 = clock64();
#endif
    bool gather = false;  // the sparse final pass is a gather from the buffers
    Cand cd{0, false, kNegInf, kNegInf};
    if (SCAN) {
      float zmax = kNegInf;
      constexpr int KT = NORM == HFAN_SPARSEMAX ? HFAN_KT_SPM : HFAN_KT_ENT;  // tracked chunk maxima (entmax15 supports are wider)
      float tk[KT];  // the KT largest chunk maxima so far (raw scores, descending)
#pragma unroll
      for (int k = 0; k < KT; ++k) tk[k] = kNegInf;
      // Every warpgroup's bound is a lower bound of the row's tau, so they
      // publish it and adopt the largest (a stale read is still a valid bound).
      volatile float* xb = xch + 6144;  // [NWG][128]
      xb[wg * 128 + row] = kNegInf;
      named_bar_sync(1, NT);
      // Every row thread runs all n_tiles iterations, also after a timed-out
      // wait (ok == false, work skipped), so the periodic votes below never
      // strand a warpgroup at its barrier.
#ifdef HFAN_DIAG
      long long dw = 0, dt = 0, da = 0, dv = 0, dc = clock64(), dn;
      long long n_vote = 0, n_heavy = 0, n_app = 0, n_chunk = 0, t_vbar = 0;
#define DIAG_LAP(acc) (dn = clock64(), acc += dn - dc, dc = dn)
#else
#define DIAG_LAP(acc) ((void)0)
#endif
      for (int t = 0; t < n_tiles; ++t) {
        if (ok) ok = load_s(t, true);
        DIAG_LAP(dw);
        if (ok) {
        // chunk maxima (8 keys each) gate the candidate appends
        // (sparsemax: and their halves gate the predicated stores)
        float cm[COLS / kCW], ch[2 * (COLS / kCW)];
        float tm = kNegInf;
#pragma unroll
        for (int c = 0; c < COLS / kCW; ++c) {
          if (NORM == HFAN_SPARSEMAX) {
            ch[2 * c] = max_n<kCW / 2>(sreg + c * kCW);
            ch[2 * c + 1] = max_n<kCW / 2>(sreg + c * kCW + kCW / 2);
            cm[c] = fmaxf(ch[2 * c], ch[2 * c + 1]);
          } else {
            cm[c] = max_n<kCW>(sreg + c * kCW);
          }
          tm = fmaxf(tm, cm[c]);
        }
        zmax = fmaxf(zmax, tm * zs);
        // A tile whose scores all lie at or below the admission bound changes
        // nothing: it has no candidate, and its chunk maxima cannot raise the
        // bound (the threshold of any set of values is at most its k-th
        // largest member, so values <= thr never yield a bound above thr).
        // Only tiles with a score above the bound somewhere in the warp (and
        // every fourth tile, to adopt the other warpgroups' bounds) update the
        // KT largest chunk maxima, the bound, and the buffers.
        const bool heavy = __any_sync(0xffffffffu, tm > cd.thr_s) || (t & 3) == 0;
#ifdef HFAN_DIAG
        n_heavy += heavy;
#pragma unroll
        for (int c = 0; c < COLS / kCW; ++c) n_chunk += __any_sync(0xffffffffu, heavy && !cd.overflow && tm > cd.thr_s && cm[c] > cd.thr_s);
#endif
        if (heavy) {
          if constexpr (KT == 4 && COLS / kCW == 4) {
            top4_merge(tk, cm);
          } else {
#pragma unroll
            for (int c = 0; c < COLS / kCW; ++c) {
              float x = cm[c];
#pragma unroll
              for (int k = 0; k < KT - 1; ++k) {  // branch-free insertion
                const float hi_ = fmaxf(tk[k], x);
                x = fminf(tk[k], x);
                tk[k] = hi_;
              }
              tk[KT - 1] = fmaxf(tk[KT - 1], x);
            }
          }
          float zk[KT];
#pragma unroll
          for (int k = 0; k < KT; ++k) zk[k] = tk[k] * zs;
          float lb = tk[0] > kNegInf ? top_bound<NORM, KT>(zk) : kNegInf;
#pragma unroll
          for (int w = 0; w < NWG; ++w) lb = fmaxf(lb, xb[w * 128 + row]);
          if (lb > cd.thr) {
            cd.thr = lb;
            cd.thr_s = raw_gate(lb, izs);
          }
        }
        DIAG_LAP(dt);
        if (heavy && !cd.overflow && tm > cd.thr_s) {
#pragma unroll
          for (int c = 0; c < COLS / kCW; ++c) {
            if (!cd.overflow && cm[c] > cd.thr_s) {
              if (cd.n > CAPW - kCW) cd = buffer_compact<NORM, IDX>(cbuf, ibuf, row, cd, CAPW, zs);
              // predicated appends: every value of a (half) chunk holding a
              // candidate is written at slot n, and n only advances past the
              // candidates.  Sparsemax gates each half chunk (its candidates
              // are sparse); entmax15's fill both halves, so it gates the chunk.
              constexpr int NHC = NORM == HFAN_SPARSEMAX ? 2 : 1;
#pragma unroll
              for (int hc = 0; hc < NHC; ++hc) {
                if (!cd.overflow && (NHC == 1 || ch[2 * c + hc] > cd.thr_s)) {
#pragma unroll
                  for (int e = hc * (kCW / NHC); e < (hc + 1) * (kCW / NHC); ++e) {
                    const float x = sreg[c * kCW + e];
                    cbuf[cd.n * 128 + row] = x * zs;
                    if (IDX) ibuf[cd.n * 128 + row] = (uint16_t)((t << JB) | (c * kCW + e));
                    cd.n += x > cd.thr_s ? 1 : 0;
#ifdef HFAN_DIAG
                    n_app += x > cd.thr_s ? 1 : 0;
#endif
                  }
                }
              }
            }
          }
        }
        // Cooperative compaction once any buffer nears capacity: the threshold
        // of all candidates of the row so far (a lower bound of tau, and a far
        // tighter one than a single warpgroup's) becomes every warpgroup's
        // admission bound, and dead entries are dropped.
        DIAG_LAP(da);
        }  // ok
        // The vote runs every fourth tile and after the last (CTA-uniform);
        // the per-warpgroup compaction above guards the tiles in between.
        // The bound is published before the vote, so that every warpgroup
        // starts the union solve from the same t0.
        xb[wg * 128 + row] = cd.thr;
        // (Sparsemax supports stay far below the capacity: no vote.)
        if (NORM != HFAN_ENTMAX15) continue;
        if ((t % HFAN_VOTE_PERIOD) != HFAN_VOTE_PERIOD - 1 && t != n_tiles - 1) continue;
#ifdef HFAN_DIAG
        const long long vb0_ = clock64();
#endif
        const bool vote_ = named_bar_or(1, NT, ok && cd.n > CAPW - HFAN_VOTE_MARGIN && !cd.overflow);
#ifdef HFAN_DIAG
        t_vbar += clock64() - vb0_;
        n_vote += vote_;
#endif
        if (vote_) {
          float t0 = cd.thr;
#pragma unroll
          for (int w = 0; w < NWG; ++w) t0 = fmaxf(t0, xb[w * 128 + row]);
          float r, sup;
          union_solve(cd, t0, ok && zmax > kNegInf, HFAN_VOTE_ITERS, &r, &sup);
          if (r > cd.thr) {
            cd.thr = r;
            cd.thr_s = raw_gate(r, izs);
          }
          if (!cd.overflow) {
            int live = 0;
            for (int e = 0; e < cd.n; ++e) {
              const float z = cbuf[e * 128 + row];
              if (z > cd.thr) {
                if (IDX) ibuf[live * 128 + row] = ibuf[e * 128 + row];
                cbuf[live++ * 128 + row] = z;
              }
            }
            cd.n = live;
            if (live > CAPW - kCompactRoom) cd.overflow = true;
          }
          xb[wg * 128 + row] = cd.thr;
        }
        DIAG_LAP(dv);
      }
#ifdef HFAN_DIAG
      if (threadIdx.x == 0) {
        DIAG_ADD(1, dw);
        DIAG_ADD(2, dt);
        DIAG_ADD(3, da);
        DIAG_ADD(4, dv);
        DIAG_ADD(16, n_vote);
        DIAG_ADD(17, t_vbar);
        DIAG_ADD(18, n_app);
        DIAG_ADD(19, n_chunk);
        DIAG_ADD(20, n_heavy);
      }
#endif
#ifdef HFAN_DIAG
      if (threadIdx.x == 0) DIAG_ADD(5, clock64() - diag_t0);
      diag_t0 = clock64();
#endif
      // merge the warpgroups: row max, best lower bound, overflow
      float* xs = xch;  // [NWG][128 rows][4]
      xs[(wg * 128 + row) * 4 + 0] = zmax;
      xs[(wg * 128 + row) * 4 + 1] = cd.thr;
      xs[(wg * 128 + row) * 4 + 2] = cd.overflow ? 1.f : 0.f;
      named_bar_sync(1, NT);
      float zrow = kNegInf, lower = kNegInf;
      bool ovf = false;
#pragma unroll
      for (int w = 0; w < NWG; ++w) {
        const float* o = xs + (w * 128 + row) * 4;
        zrow = fmaxf(zrow, o[0]);
        lower = fmaxf(lower, o[1]);
        ovf |= o[2] != 0.f;
      }
      named_bar_sync(1, NT);
      // Exact tau on the union of the row's buffers.
      const bool empty = !(zrow > kNegInf);
      if (NORM == HFAN_SPARSEMAX && !empty && !ovf) {
        // Entries at or below the merged bound (a lower bound of tau) are not
        // in the support: drop them once, in order, so that the solve's
        // iterations and the gather walk only live entries (the sums, taken
        // over z > t in buffer order, are unchanged).  Sparsemax only: its
        // buffers are never compacted by votes (entmax15's are, and the
        // extra pass measured slower there).
        int live = 0;
        for (int e = 0; e < cd.n; ++e) {
          const float z = cbuf[e * 128 + row];
          if (z > lower) {
            if (IDX) ibuf[live * 128 + row] = ibuf[e * 128 + row];
            cbuf[live++ * 128 + row] = z;
          }
        }
        cd.n = live;
      }
      bool pending = !empty && ovf;  // overflowing rows go to whole-row sweeps
      float tsol = lower;
      if (union_solve(cd, lower, !empty && !ovf, 64, &tsol, &support, true, zrow)) {
        tau = tsol;
      } else if (!empty && !ovf) {
        pending = true;  // did not converge: sweep the row
      }
      if (empty) tau = kPosInf;  // no visible key: zero row
      if (pending) {
        tau = kPosInf;
        lower = fmaxf(lower, tsol);
      }
      for (int sweep = 0;; ++sweep) {
        // CTA-wide decision (uniform across the row threads): another
        // bracket sweep, or the final pass.  The candidate buffers were
        // written through the generic proxy and the final pass's TMA loads
        // overwrite them: order the two.
        fence_proxy_async_smem();
        named_bar_sync(1, NT);
        if (threadIdx.x == 0) ctl->any_pending = 0;
        named_bar_sync(1, NT);
        if (pending) ctl->any_pending = 1;
        if (!ok) ctl->abort = 1;
        named_bar_sync(1, NT);
        if (threadIdx.x == 0) {
          const bool more_ = ctl->any_pending != 0 && sweep < kMaxSweeps && ctl->abort == 0;
          // Without sweeps every row's support is in its candidate buffers
          // (every score above the final bound was buffered), so P V is
          // gathered from them; rows settled by sweeps need the full pass.
          const bool gather_ok = IDX && !DROP && sweep == 0 && ctl->any_pending == 0 && ctl->abort == 0 &&
                                 n_tiles <= (65536 >> JB);
          ctl->next_pass = more_ ? kPassSweep : (gather_ok ? kPassGather : kPassFinal);
          DIAG_ADD(10, gather_ok && !more_ ? 1 : 0);
          DIAG_ADD(11, more_ ? 1 : 0);
          mbar_arrive(&bars->ctrl);
        }
        named_bar_sync(1, NT);
        gather = ctl->next_pass == kPassGather;
        if (ctl->next_pass != kPassSweep) break;
        // Besides the sums above the bound, a pending row buffers every
        // score above it again: once they fit (the bound is close to tau),
        // the exact solve on the buffers ends the row's sweeps.
        // (Only rows whose previous count above the bound suggests they fit.)
        TauStats st{0.f, 0.f, 0.f, kPosInf};
        cd.n = 0;
        const bool refill = __any_sync(0xffffffffu, pending && sweep > 0 && support <= 0.75f * CAPW * NWG);
        for (int t = 0; t < n_tiles && ok; ++t) {
          if (!(ok = load_s(t, true))) break;
          if (pending) {
            if (refill) {
#pragma unroll
              for (int j = 0; j < COLS; ++j) {
                const float z = sreg[j] * zs;
                tau_accumulate_ref(st, z, lower, zrow);
                if (z > lower) {
                  if (cd.n < CAPW) cbuf[cd.n * 128 + row] = z;
                  ++cd.n;
                }
              }
            } else {
              cd.n = CAPW + 1;
#pragma unroll
              for (int j = 0; j < COLS; ++j) tau_accumulate_ref(st, sreg[j] * zs, lower, zrow);
            }
          }
        }
        volatile float* xo = xch + 6144;  // [NWG][128]: this warpgroup's buffer overflowed
        xo[wg * 128 + row] = cd.n > CAPW ? 1.f : 0.f;
        // combine the warpgroups' sums; all then take the same step
        float* xt = xch;  // [NWG][128 rows][4], free again once the merge above was read
        xt[(wg * 128 + row) * 4 + 0] = st.cnt;
        xt[(wg * 128 + row) * 4 + 1] = st.s1;
        xt[(wg * 128 + row) * 4 + 2] = st.s2;
        xt[(wg * 128 + row) * 4 + 3] = st.zmin;
        named_bar_sync(1, NT);
        TauStats all{0.f, 0.f, 0.f, kPosInf};
#pragma unroll
        for (int w = 0; w < NWG; ++w) {
          const float* o = xt + (w * 128 + row) * 4;
          all.cnt += o[0];
          all.s1 += o[1];
          all.s2 += o[2];
          all.zmin = fminf(all.zmin, o[3]);
        }
        bool fits = pending && ok;
#pragma unroll
        for (int w = 0; w < NWG; ++w) fits = fits && xo[w * 128 + row] == 0.f;
        named_bar_sync(1, NT);
        float tb, sb;
        if (union_solve(cd, lower, fits, 64, &tb, &sb, true, zrow)) {
          tau = tb;
          support = sb;
          pending = false;
        } else if (pending && ok) {
          support = all.cnt;
          pending = !tau_step_ref(NORM, all, zrow, &lower, &tau);
        }
      }
    }

#ifdef HFAN_DIAG
    if (threadIdx.x == 0) DIAG_ADD(6, clock64() - diag_t0);
    diag_t0 = clock64();
#endif
    // ---- sparse gather (kPassGather): O = sum_j p_j v_j and U = sum_j w_j v_j
    // over the support entries of the candidate buffers, instead of a second
    // Q K^T and a P V over every key tile.  Each thread first keeps the
    // support of its own buffer in place (d = z - tau > 0 and the key) and
    // sets the tile bits; then every warpgroup walks the NWG lists of its row
    // for its 32 head-dim columns, reading V rows from global memory (L2).
    // The order of the sums is fixed: buffer order (key order within a
    // warpgroup), then warpgroup order.
    auto gather_pv = [&](float tau_) {
      int* xn = reinterpret_cast<int*>(xch + 6144);  // [NWG][128] list lengths
      const T* vb = static_cast<const T*>(p.v) + key_off(p, b, kvh, 0, p.v_sb, p.v_sh, p.v_st);
      auto vrow = [&](int w, int id) -> const T* {
        const int key = k_lo + (id >> JB) * kBN + w * COLS + (id & (COLS - 1));
        const int64_t tok = varlen ? (int64_t)(g.k_start + key) : (int64_t)key;
        return vb + tok * p.v_st;
      };
      int m = 0;
      const int64_t srow = (int64_t)g.q_start + i;  // stats row
      for (int e = 0; e < cd.n; ++e) {
        const float z = cbuf[e * 128 + row];
        if (z > tau_) {
          const uint16_t id = ibuf[e * 128 + row];
          cbuf[m * 128 + row] = z - tau_;
          ibuf[m * 128 + row] = id;
          if (lists && row_ok && m < kSupSlots / NWG) {
            const int key = k_lo + (id >> JB) * kBN + wg * COLS + (id & (COLS - 1));
            const float d = z - tau_, pr = NORM == HFAN_SPARSEMAX ? d : d * d;
            p.sl_ent[((int64_t)h * p.rows_total + srow) * kSupSlots + wg * (kSupSlots / NWG) + m] =
                make_int2(varlen ? g.k_start + key : key, __float_as_int(pr));
          }
          ++m;
          // the four warpgroups read this V row next: bring it into L2 now
          const T* vr = vrow(wg, id);
#pragma unroll
          for (int c = 0; c < HD * (int)sizeof(T); c += 128) prefetch_l2(reinterpret_cast<const char*>(vr) + c);
          if (track) {
            const int kt = kt0 + (id >> JB);
            atomicOr(&sbits[(row >> 6) * kMaskWordsMax + (kt >> 5)], 1u << (kt & 31));
          }
        }
      }
      xn[wg * 128 + row] = m;
      if (lists && row_ok) {
        p.sl_cnt[((int64_t)h * p.rows_total + srow) * NWG + wg] = min(m, kSupSlots / NWG);
        if (m > kSupSlots / NWG) atomicExch(p.sl_flag, 1);  // the backward runs the tile kernels
      }
      named_bar_sync(1, NT);
      uint64_t acc[16], accu[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = accu[j] = 0ull;
      float wsum_ = 0.f;
      for (int w = 0; w < NWG; ++w) {
        const int mw = xn[w * 128 + row];
        const float* db = cbuf0 + w * CAPW * 128;
        const uint16_t* ib = ibuf0 + w * CAPW * 128;
        for (int e = 0; e < mw; ++e) {
          const float d = db[e * 128 + row];
          const uint4* vp = reinterpret_cast<const uint4*>(vrow(w, ib[e * 128 + row]) + wg * 32);
          // p = d (sparsemax) or d^2 (entmax15); w = 1[p > 0] or d
          const float pr = NORM == HFAN_SPARSEMAX ? d : d * d;
          const float wt = NORM == HFAN_SPARSEMAX ? 1.f : d;
          wsum_ += wt;
          const uint64_t p2 = f2_pack(pr, pr), w2 = f2_pack(wt, wt);
          uint4 x[4];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) x[q4] = __ldg(vp + q4);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint32_t xs[4] = {x[q4].x, x[q4].y, x[q4].z, x[q4].w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const uint64_t v2 = unpack2<BF16>(xs[r]);
              acc[q4 * 4 + r] = ffma2(p2, v2, acc[q4 * 4 + r]);
              if (want_u) accu[q4 * 4 + r] = ffma2(w2, v2, accu[q4 * 4 + r]);
            }
          }
        }
      }
      if (row_ok) {
        auto put = [&](T* dst, const uint64_t (&a)[16], float inv) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 v;
            v.x = pack2<BF16>(f2_lo(a[q4 * 4 + 0]) * inv, f2_hi(a[q4 * 4 + 0]) * inv);
            v.y = pack2<BF16>(f2_lo(a[q4 * 4 + 1]) * inv, f2_hi(a[q4 * 4 + 1]) * inv);
            v.z = pack2<BF16>(f2_lo(a[q4 * 4 + 2]) * inv, f2_hi(a[q4 * 4 + 2]) * inv);
            v.w = pack2<BF16>(f2_lo(a[q4 * 4 + 3]) * inv, f2_hi(a[q4 * 4 + 3]) * inv);
            reinterpret_cast<uint4*>(dst)[q4] = v;
          }
        };
        put(static_cast<T*>(p.o) + qrow_off(p, g, b, h, i, p.o_sb, p.o_sh, p.o_st) + wg * 32, acc, 1.f);
        if (want_u)
          put(static_cast<T*>(p.wm) + qrow_off(p, g, b, h, i, p.wm_sb, p.wm_sh, p.wm_st) + wg * 32, accu,
              wsum_ > 0.f ? 1.f / wsum_ : 0.f);
      }
    };

    // ---- final pass: P and O
    float m_ref = 0.f, l = wg == 0 ? 1.f : 0.f;  // the implicit zero logit counts once
    const float ntau = -tau;
    // Dropout: P V uses p * keep / (1 - p_drop); the softmax1 denominator and
    // the sparse thresholds use the undropped probabilities.
    constexpr bool drop = DROP;  // a separate instantiation: no cost without dropout
    uint32_t seed_lo = 0u, seed_hi = 0u;
    uint64_t drow = 0;
    if (drop) {
      const uint64_t sd = (uint64_t)*p.drop_seed;
      seed_lo = (uint32_t)sd;
      seed_hi = (uint32_t)(sd >> 32);
      drow = ((uint64_t)b * p.hq + h) * p.len_q + (row_ok ? i : 0);
    }
    // softmax1 meets a named barrier on every tile, so after a timeout the loop
    // keeps running (with the work skipped) instead of leaving it.
#ifdef HFAN_DIAG
    long long dg_s = 0, dg_pv = 0, dg_c = 0, dg_st = 0, dgc0 = 0;
#endif
    float wsum = 0.f;  // sparse: sum_j w_j of this warpgroup's keys (U's normaliser)
    int sl_n = 0;      // entries of this warpgroup's support sub-list
    const int64_t sl_row = (int64_t)g.q_start + i;
    for (int t = 0; t < (gather ? 0 : n_tiles) && (ok || !SPARSE); ++t) {
      if (ok) DIAG_T(dg_s, ok = load_s(t, false));
#ifdef HFAN_DIAG
      dgc0 = clock64();
#endif
      uint32_t wpk[COLS / 2];  // sparse with U: packed W of this warpgroup's keys
      float alpha = 1.f;
      bool rescale = false;
      if (!SPARSE) {
        // log2 units: x = s * scale * log2(e); the row max over all warpgroups
        float tmax = max_n<COLS>(sreg) * zs;
        float* xm = xch + (t & 1) * (NWG * 128);  // double-buffered by tile parity: one barrier per tile
        xm[wg * 128 + row] = tmax;
        named_bar_sync(1, NT);
#pragma unroll
        for (int w = 0; w < NWG; ++w) tmax = fmaxf(tmax, xm[w * 128 + row]);
        if (tmax > m_ref + kRescaleLog2) {
          alpha = exp2f(m_ref - tmax);
          m_ref = tmax;
          l *= alpha;
          rescale = t > 0;
        }
        const uint64_t zs2 = f2_pack(zs, zs), nm2 = f2_pack(-m_ref, -m_ref);
        uint64_t l2 = 0;
#pragma unroll
        for (int j = 0; j < COLS; j += 2) {
          const uint64_t x = ffma2(f2_pack(sreg[j], sreg[j + 1]), zs2, nm2);
          const float e0 = ex2_ftz(f2_lo(x)), e1 = ex2_ftz(f2_hi(x));  // exp2(-inf) = 0 for masked keys
          sreg[j] = e0;
          sreg[j + 1] = e1;
          l2 = fadd2(l2, f2_pack(e0, e1));
        }
        l += f2_lo(l2) + f2_hi(l2);
      } else {
        const uint64_t zs2 = f2_pack(zs, zs), nt2 = f2_pack(ntau, ntau);
        // keep bits of this warpgroup's COLS keys (bit j = key kb + j)
        uint64_t kbits = ~0ull;
        if (drop) {
          const int kb = k_lo + t * kBN + wg * COLS;  // a multiple of 4: groups of four keys
          kbits = 0ull;
#pragma unroll
          for (int g4 = 0; g4 < COLS / 4; ++g4)
            kbits |= (uint64_t)dropout_keep4(drow, (uint32_t)((kb >> 2) + g4), seed_lo, seed_hi, p.drop_thr24)
                     << (4 * g4);
        }
        uint64_t ws2 = 0;  // sum of w over the pairs (undropped)
        bool nzl = false;  // dropout: some undropped p > 0 (the mask is about p, not the kept values)
#pragma unroll
        for (int j = 0; j < COLS; j += 2) {
          uint64_t d = ffma2(f2_pack(sreg[j], sreg[j + 1]), zs2, nt2);
          d = f2_pack(fmaxf(f2_lo(d), 0.f), fmaxf(f2_hi(d), 0.f));
          // w = dp/dz up to the constant the backward folds in: 1[p > 0] or (z - tau)_+
          uint64_t w = NORM == HFAN_SPARSEMAX ? f2_pack(f2_lo(d) > 0.f ? 1.f : 0.f, f2_hi(d) > 0.f ? 1.f : 0.f) : d;
          if (drop && track) nzl |= (f2_lo(d) > 0.f) | (f2_hi(d) > 0.f);
          if (NORM != HFAN_SPARSEMAX) d = fmul2(d, d);
          if (want_u) {
            ws2 = fadd2(ws2, w);
            if (drop) {
              const uint64_t ks = f2_pack(((kbits >> j) & 1ull) ? p.drop_scale : 0.f,
                                          ((kbits >> (j + 1)) & 1ull) ? p.drop_scale : 0.f);
              w = fmul2(w, ks);
            }
            wpk[j / 2] = pack2<BF16>(f2_lo(w), f2_hi(w));
          }
          if (drop) {
            d = fmul2(d, f2_pack(((kbits >> j) & 1ull) ? p.drop_scale : 0.f,
                                 ((kbits >> (j + 1)) & 1ull) ? p.drop_scale : 0.f));
          }
          sreg[j] = f2_lo(d);
          sreg[j + 1] = f2_hi(d);
        }
        wsum += f2_lo(ws2) + f2_hi(ws2);
        if (want_u && ok) {
          // P, then W, over this warpgroup's own COLS columns of the S buffer
          // the tile came from (read into registers above; nobody else reads
          // them, and the buffer is reissued only after this tile's P V).
          // Issued before the support lists and tile bits are worked out, so
          // that the stores are in flight meanwhile.
          const uint32_t sl = tmem + lane_addr + ((sc - 1) & 1) * 128 + wg * COLS;
#pragma unroll
          for (int c = 0; c < COLS / 32; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[j] = pack2<BF16>(sreg[c * 32 + 2 * j], sreg[c * 32 + 2 * j + 1]);
            tmem_st16(sl + c * 16, pk);
            tmem_st16(sl + COLS / 2 + c * 16, *reinterpret_cast<uint32_t(*)[16]>(wpk + c * 16));
          }
        }
        if (lists && row_ok) {
          // this warpgroup's keys with p > 0, in key order, into the row's
          // sub-list (8-key chunks gate the predicated appends)
          const int kb = (varlen ? g.k_start : 0) + k_lo + t * kBN + wg * COLS;
          int2* base = p.sl_ent + ((int64_t)h * p.rows_total + sl_row) * kSupSlots + wg * (kSupSlots / NWG);
#pragma unroll
          for (int c = 0; c < COLS / 8; ++c) {
            if (max_n<8>(sreg + c * 8) > 0.f) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (sreg[c * 8 + e] > 0.f) {
                  if (sl_n < kSupSlots / NWG) base[sl_n] = make_int2(kb + c * 8 + e, __float_as_int(sreg[c * 8 + e]));
                  ++sl_n;
                }
              }
            }
          }
        }
        if (track) {  // this warp's 32 rows x COLS keys: any p > 0 sets the tile's bit for its 64-row half
          const unsigned bal = __ballot_sync(0xffffffffu, drop ? nzl : max_n<COLS>(sreg) > 0.f);
          const int kt = kt0 + t;
          if (lane == 0 && bal != 0u)
            atomicOr(&sbits[((warp & 3) >> 1) * kMaskWordsMax + (kt >> 5)], 1u << (kt & 31));
        }
      }
      if (drop && !SPARSE) {
        const int kb = k_lo + t * kBN + wg * COLS;  // a multiple of 4: groups of four keys
#pragma unroll
        for (int g4 = 0; g4 < COLS / 4; ++g4) {
          const uint32_t keep = dropout_keep4(drow, (uint32_t)((kb >> 2) + g4), seed_lo, seed_hi, p.drop_thr24);
#pragma unroll
          for (int e = 0; e < 4; ++e) sreg[4 * g4 + e] *= ((keep >> e) & 1u) ? p.drop_scale : 0.f;
        }
      }
      if (!ok) continue;
      // O may be rescaled once every earlier P V has completed; P buffer pb
      // is free once the P V two tiles back (its last reader) has.
#ifdef HFAN_DIAG
      { const long long n_ = clock64(); dg_c += n_ - dgc0; dgc0 = n_; }
#endif
      const int pb = pc & 1;
      if (__any_sync(0xffffffffu, rescale)) {
        if (!(ok = wait_warp(&bars->pv_done[(pc - 1) & 1], ((pc - 1) >> 1) & 1, abort_flag))) continue;
        tc_fence_after();
        // warp-collective: lanes without a rescale multiply by one
        const float f = rescale ? alpha : 1.f;
        uint32_t r[32];
        tmem_ld32(tmem_o + lane_addr + wg * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * f);
        tmem_st32(tmem_o + lane_addr + wg * 32, r);
        tmem_wait_st();
      }
      if (!want_u) {
        if (pc >= 2) {
          DIAG_T(dg_pv, ok = wait_warp(&bars->pv_done[pb], ((pc >> 1) & 1) ^ 1, abort_flag));
          if (!ok) continue;
          tc_fence_after();
        }
        // this warpgroup's COLS keys of the P row -> TMEM columns
        // [COLS/2 wg, COLS/2 (wg + 1)) of buffer pb, packed in key order
#pragma unroll
        for (int c = 0; c < COLS / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = pack2<BF16>(sreg[c * 32 + 2 * j], sreg[c * 32 + 2 * j + 1]);
          tmem_st16(tmem_p + lane_addr + pb * 64 + wg * (COLS / 2) + c * 16, pk);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      warp_arrive(&bars->p_full[pb]);
      ++pc;
#ifdef HFAN_DIAG
      dg_st += clock64() - dgc0;
#endif
    }
    if (lists && row_ok && !gather) {
      p.sl_cnt[((int64_t)h * p.rows_total + sl_row) * NWG + wg] = min(sl_n, kSupSlots / NWG);
      if (sl_n > kSupSlots / NWG) atomicExch(p.sl_flag, 1);
    }
    if (ok && n_tiles > 0 && !gather) {
      // with U: the last tile's P V was committed to the barrier of its S buffer
      const int lb = want_u ? (int)((sc - 1) & 1u) : (int)((pc - 1) & 1u);
      ok = wait_warp(&bars->pv_done[lb], ((pc - 1) >> 1) & 1, abort_flag);
      tc_fence_after();
    }
#ifdef HFAN_DIAG
    if (threadIdx.x == 0) {
      DIAG_ADD(7, clock64() - diag_t0);
      DIAG_ADD(12, dg_s);
      DIAG_ADD(13, dg_pv);
      DIAG_ADD(22, dg_c);
      DIAG_ADD(23, dg_st);
      DIAG_ADD(8, dls_w);
      DIAG_ADD(9, dls_l);
    }
#endif
    if (!ok) record_error(p, ctl, kDevWaitTimeout);
    if (SPARSE && IDX && !DROP && gather) {
#ifdef HFAN_DIAG
      const long long g0_ = clock64();
#endif
      gather_pv(tau);
#ifdef HFAN_DIAG
      if (threadIdx.x == 0) DIAG_ADD(14, clock64() - g0_);
#endif
    }
    if (SPARSE && track && p.tile_mask != nullptr) {
      named_bar_sync(1, NT);  // every row warp's support bits are in
      if (threadIdx.x < 2 * p.mask_words) {
        const int half = threadIdx.x / p.mask_words, w = threadIdx.x % p.mask_words;
        p.tile_mask[((int64_t)(h * p.batch + b) * p.mask_qb + 2 * qt + half) * p.mask_words + w] =
            sbits[half * kMaskWordsMax + w];
      }
    }
    if (!gather && (!SPARSE || want_u)) {
      // total denominator of the row (softmax1) or sum_j w_j (sparse, U)
      float* xl = xch + 2 * NWG * 128;
      xl[wg * 128 + row] = SPARSE ? wsum : l;
      named_bar_sync(1, NT);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < NWG; ++w) tot += xl[w * 128 + row];
      if (SPARSE) wsum = tot;
      else l = tot;
    }

    // ---- epilogue: this warpgroup's 32 columns of the O row -> global, row
    // statistics.  The TMEM load is warp-collective, so every lane loads; only
    // valid rows store.
    if (!gather) {
      const float inv = SPARSE ? 1.f : 1.f / l;
      T* orow = static_cast<T*>(p.o) + qrow_off(p, g, b, h, row_ok ? i : 0, p.o_sb, p.o_sh, p.o_st);
      uint32_t r[32];
      const int col = wg * 32;
      if (n_tiles > 0) {
        tmem_ld32(tmem_o + lane_addr + col, r);
        tmem_wait_ld();
      }
      if (n_tiles == 0 || !ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(r[j + 0]) * inv, __uint_as_float(r[j + 1]) * inv);
          v.y = pack2<BF16>(__uint_as_float(r[j + 2]) * inv, __uint_as_float(r[j + 3]) * inv);
          v.z = pack2<BF16>(__uint_as_float(r[j + 4]) * inv, __uint_as_float(r[j + 5]) * inv);
          v.w = pack2<BF16>(__uint_as_float(r[j + 6]) * inv, __uint_as_float(r[j + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + col + j) = v;
        }
      }
    }
    if (want_u && !gather) {
      // this warpgroup's 32 columns of wmean = U / sum_j w_j
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
      T* wrow = static_cast<T*>(p.wm) + qrow_off(p, g, b, h, row_ok ? i : 0, p.wm_sb, p.wm_sh, p.wm_st);
      uint32_t r[32];
      const int col = wg * 32;
      if (n_tiles > 0) {
        tmem_ld32(tmem_u + lane_addr + col, r);
        tmem_wait_ld();
      }
      if (n_tiles == 0 || !ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(r[j + 0]) * inv, __uint_as_float(r[j + 1]) * inv);
          v.y = pack2<BF16>(__uint_as_float(r[j + 2]) * inv, __uint_as_float(r[j + 3]) * inv);
          v.z = pack2<BF16>(__uint_as_float(r[j + 4]) * inv, __uint_as_float(r[j + 5]) * inv);
          v.w = pack2<BF16>(__uint_as_float(r[j + 6]) * inv, __uint_as_float(r[j + 7]) * inv);
          *reinterpret_cast<uint4*>(wrow + col + j) = v;
        }
      }
    }
    if (row_ok && wg == 0) {
      const int64_t si = stat_index(p, g, h, i);
      if (SPARSE) {
        p.stats[si] = tau;
        p.stats[(int64_t)p.hq * p.rows_total + si] = support;
      } else {
        p.stats[si] = m_ref;
        p.stats[(int64_t)p.hq * p.rows_total + si] = l;
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

// ------------------------------------------------------------------ host
template <int HD, bool BF16>
cudaError_t launch_fwd(const AttnParams& p, int max_q, cudaStream_t stream) {
  const bool varlen = p.cu_q != nullptr;
  CUtensorMap tq, tk, tv;
  // Token extent: dense maps cover one sequence (rows past it read as zero);
  // packed varlen maps cover all packed rows.
  const int64_t tq_n = varlen ? p.rows_total : p.len_q;
  const int64_t tk_n = varlen ? p.rows_k : p.len_k;
  const int batch = varlen ? 1 : p.batch;
  const int64_t q_sb = varlen ? tq_n * p.q_st : p.q_sb;
  const int64_t k_sb = varlen ? tk_n * p.k_st : p.k_sb;
  const int64_t v_sb = varlen ? tk_n * p.v_st : p.v_sb;
  if (!make_map(&tq, p.q, BF16, HD, tq_n, p.hq, batch, p.q_st, p.q_sh, q_sb) ||
      !make_map(&tk, p.k, BF16, HD, tk_n, p.hkv, batch, p.k_st, p.k_sh, k_sb) ||
      !make_map(&tv, p.v, BF16, HD, tk_n, p.hkv, batch, p.v_st, p.v_sh, v_sb))
    return cudaErrorInvalidValue;
  const size_t smem = Layout<HD>::TOTAL;
  dim3 grid((max_q + kBM - 1) / kBM, p.hq, p.batch);
  AttnParams pl = p;  // query tiles re-read K and V
  pl.tile_lpt = (varlen ? tk_n : (int64_t)p.batch * tk_n) * p.hkv * HD * 4 <= kLptMaxReread;
  auto go = [&](auto kernel) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    kernel<<<grid, Roles<HD, 2>::THREADS, smem, stream>>>(tq, tk, tv, pl);
    return cudaSuccess;
  };
  const bool drop = p.drop_thr24 != 0u;
  cudaError_t e;
  switch (p.norm) {
    case HFAN_SOFTMAX1:
      e = drop ? go(tc_fwd_kernel<HD, BF16, HFAN_SOFTMAX1, true>) : go(tc_fwd_kernel<HD, BF16, HFAN_SOFTMAX1, false>);
      break;
    case HFAN_SPARSEMAX:
      e = drop ? go(tc_fwd_kernel<HD, BF16, HFAN_SPARSEMAX, true>) : go(tc_fwd_kernel<HD, BF16, HFAN_SPARSEMAX, false>);
      break;
    default:
      e = drop ? go(tc_fwd_kernel<HD, BF16, HFAN_ENTMAX15, true>) : go(tc_fwd_kernel<HD, BF16, HFAN_ENTMAX15, false>);
      break;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

bool tc_supported(int dtype, const AttnParams& p) {
  if (dtype != HFAN_BFLOAT16 && dtype != HFAN_FLOAT16) return false;
  if (p.paged) return false;
  if (p.d != 64 && p.d != 128) return false;
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) || !aligned16(p.o)) return false;
  if (!stride_ok(p.q_st) || !stride_ok(p.q_sh) || !stride_ok(p.k_st) || !stride_ok(p.k_sh) ||
      !stride_ok(p.v_st) || !stride_ok(p.v_sh) || (p.o_st % 8) != 0 || (p.o_sh % 8) != 0)
    return false;
  if (p.cu_q == nullptr) {
    if ((p.batch > 1) && (!stride_ok(p.q_sb) || !stride_ok(p.k_sb) || !stride_ok(p.v_sb))) return false;
    if (p.batch > 1 && (p.o_sb % 8) != 0) return false;
  } else {
    if (p.rows_k <= 0) return false;  // packed key rows bound the K/V maps
  }
  return true;
}

cudaError_t tc_attention_fwd(int dtype, const AttnParams& p, int max_q, cudaStream_t s) {
  const bool bf16 = dtype == HFAN_BFLOAT16;
  if (p.d == 128) return bf16 ? launch_fwd<128, true>(p, max_q, s) : launch_fwd<128, false>(p, max_q, s);
  return bf16 ? launch_fwd<64, true>(p, max_q, s) : launch_fwd<64, false>(p, max_q, s);
}


}  // namespace hfan
