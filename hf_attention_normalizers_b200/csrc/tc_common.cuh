// Helpers shared by the tensor-core forward and backward kernels: warp-uniform
// bounded waits, 16-bit packing, and host-side TMA tensor-map construction.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "params.cuh"
#include "tc_ptx.cuh"

namespace hfan {
namespace tc {

constexpr uint32_t kHalf = 128u * 128u;  // one 128-row x 128-byte swizzled half tile

// Wait whose outcome is uniform across the warp, so that the warp-collective
// tcgen05.ld / tcgen05.st that follow are executed by all 32 lanes or none.
__device__ __forceinline__ bool wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort) {
  bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// Arrival of a whole warp on a barrier initialised with one count per warp:
// every lane has finished (and fenced) its own accesses before the call, the
// warp converges, and lane 0 arrives.  Row-to-MMA barriers count warps, not
// threads, so that their completion is not serialised behind hundreds of
// shared-memory arrivals.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// ---- per-element arithmetic of the row warps (their issue slots bound the
// kernels): three-input max, packed f32x2 FMA/MUL/ADD, and the hardware
// base-2 exponential (denormal results flush to zero; P is stored as 16-bit
// values whose smallest normal is 2^-126 (bf16) or 2^-14 (fp16) anyway).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Maximum of N values as a tree of three-input maxima.
template <int N>
__device__ __forceinline__ float max_n(const float* v) {
  if constexpr (N == 1) {
    return v[0];
  } else if constexpr (N == 2) {
    return fmaxf(v[0], v[1]);
  } else if constexpr (N == 3) {
    return max3f(v[0], v[1], v[2]);
  } else {
    constexpr int A = (N + 2) / 3, B = (N - A + 1) / 2;
    return max3f(max_n<A>(v), max_n<B>(v + A), max_n<N - A - B>(v + A + B));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// P (or dS) row r of a 128 x 128 16-bit tile -> shared memory, K-major with
// 128-byte swizzle: two 64-column halves kHalf apart; 16-byte chunk c of row
// r sits at chunk position c ^ (r & 7).  `pk` holds the row as 64 packed pairs.
__device__ __forceinline__ void store_row_sw128(uint8_t* base, int row, const uint32_t (&pk)[64]) {
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    const int hh = c >> 3, cc = c & 7;
    uint4 v = make_uint4(pk[c * 4 + 0], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
    *reinterpret_cast<uint4*>(base + hh * kHalf + row * 128 + ((cc ^ (row & 7)) << 4)) = v;
  }
}

// One 64-column half (hh = 0 or 1) of such a row: 32 packed pairs.
__device__ __forceinline__ void store_half_sw128(uint8_t* base, int hh, int row, const uint32_t (&pk)[32]) {
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 v = make_uint4(pk[c * 4 + 0], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
    *reinterpret_cast<uint4*>(base + hh * kHalf + row * 128 + ((c ^ (row & 7)) << 4)) = v;
  }
}

// NCH consecutive 16-byte chunks (8 columns each), starting at chunk c0 of a
// 16-chunk (128-column) row, from packed pairs pk[4 * NCH].
template <int NCH>
__device__ __forceinline__ void store_chunks_sw128(uint8_t* base, int row, int c0, const uint32_t* pk) {
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int chunk = c0 + c, hh = chunk >> 3, cc = chunk & 7;
    uint4 v = make_uint4(pk[c * 4 + 0], pk[c * 4 + 1], pk[c * 4 + 2], pk[c * 4 + 3]);
    *reinterpret_cast<uint4*>(base + hh * kHalf + row * 128 + ((cc ^ (row & 7)) << 4)) = v;
  }
}

// Warp roles of the tensor-core kernels: HD / 32 row warpgroups (warpgroup wg
// owns 128 / NWG columns of each 128 x 128 tile and 32 head-dim columns),
// then one TMA warp and one MMA warp.
template <int HD, int ISSUERS = 1>
struct Roles {
  static constexpr int NWG = HD / 32;
  static constexpr int ROW_THREADS = 128 * NWG;
  static constexpr int TMA_WARP = 4 * NWG;
  static constexpr int MMA_WARP = 4 * NWG + 1;
  static constexpr int MMA2_WARP = 4 * NWG + 2;  // second MMA issuer (kernels with ISSUERS == 2)
  static constexpr int THREADS = 32 * (4 * NWG + 1 + ISSUERS);
};

// ------------------------------------------------------------------ host
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 4-D map (dim, token, head, batch) with a 64 x 128 x 1 x 1 box, 128-byte swizzle.
inline bool make_map(CUtensorMap* m, const void* base, bool bf16, int d, int64_t tokens, int heads, int batch,
              int64_t st, int64_t sh, int64_t sb, int box_rows = 128) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  // The encoder is a driver call and needs a current context.  A thread that
  // has made no runtime call yet (for example autograd's backward worker, when
  // nothing ran on it before this library) has none: cudaFree(nullptr) binds
  // the current device's primary context and does nothing else.
  cudaFree(nullptr);
  cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)tokens, (cuuint64_t)heads, (cuuint64_t)batch};
  cuuint64_t strides[3] = {(cuuint64_t)st * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }
inline bool stride_ok(int64_t s) { return s > 0 && (s % 8) == 0 && s < ((int64_t)1 << 38); }


// Tile coordinates of this CTA.  Blocks are dispatched in increasing linear
// id (x fastest).  In the default order every (head, batch) column of tiles
// is handed out whole, so on a grid of a few waves the heaviest tiles of the
// last heads start late and the kernel ends on a long tail.  With `lpt` the
// tile index x becomes the slowest-varying coordinate: all heads' tiles of
// one weight class are handed out before any lighter class (longest
// processing time first list scheduling; heads of one KV group stay
// adjacent).  That spreads the CTAs in flight over every head, so the host
// enables it only when the operand that CTAs re-read from L2 is small.
__device__ __forceinline__ uint3 tile_coords(int lpt) {
  if (!lpt) return make_uint3(blockIdx.x, blockIdx.y, blockIdx.z);
  const unsigned yz = gridDim.y * gridDim.z;
  const unsigned lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const unsigned r = lin % yz;
  return make_uint3(lin / yz, r % gridDim.y, r / gridDim.y);
}

// Longest-first order is allowed when the re-read operand (K/V for query
// tiles, Q/dO for key tiles) fits in about a third of L2.
constexpr int64_t kLptMaxReread = 40ll << 20;

// Key-tile support bitmask (sparse normalizers): words per 64-row block.
// 32 words track 1024 key tiles (131072 keys); longer rows run without it.
constexpr int kMaskWordsMax = 32;

// Walks the set bits of bits[0 ..] in increasing order (all of 0 .. n - 1
// when bits is null); next() returns n once they are exhausted.
struct BitWalk {
  const uint32_t* bits;
  int n, word, cur;
  uint32_t rest;
  __device__ __forceinline__ BitWalk(const uint32_t* b, int n_) : bits(b), n(n_), word(-1), cur(-1), rest(0u) {}
  __device__ __forceinline__ int next() {
    if (bits == nullptr) return cur = min(cur + 1, n);
    while (rest == 0u) {
      if (++word * 32 >= n) return n;
      rest = bits[word];
    }
    const int u = word * 32 + __ffs(rest) - 1;
    rest &= rest - 1u;
    return u;
  }
};


}  // namespace tc
}  // namespace hfan
