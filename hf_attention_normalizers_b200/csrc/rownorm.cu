// Row normalizers on a materialised [rows, n] score matrix (last axis).
//
// These are the CUDA counterparts of the reference's eager autograd Functions
// (vutils/softmax1.py:4-21, vutils/entmax.py:136-183).  They serve the paths
// that must materialise scores -- an arbitrary attention mask -- and the
// standalone ``softmax_1`` / ``sparsemax`` / ``entmax15`` functions.  One warp
// per row; the sparse thresholds use the exact bracket + closed-form solve of
// common.cuh (no sort).
#include "common.cuh"

namespace hfan {

template <typename T, int NORM>
__global__ void __launch_bounds__(256) rownorm_fwd_kernel(int64_t rows, int64_t n, const T* x,
                                                          int64_t ldx, T* y, int64_t ldy) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * ldx;
  T* yr = y + row * ldy;
  float xmax = kNegInf;
  for (int64_t j = lane; j < n; j += 32) xmax = fmaxf(xmax, to_f32<T>(xr[j]));
  xmax = warp_max(xmax);
  if (NORM == HFAN_SOFTMAX1) {
    // exp(x - m) / (sum exp(x - m) + exp(-m)), with m = max(xmax, 0) so that
    // neither term overflows (same value as vutils/softmax1.py:11-21).
    float m = fmaxf(xmax, 0.f);
    float l = 0.f;
    for (int64_t j = lane; j < n; j += 32) l += expf(to_f32<T>(xr[j]) - m);
    l = warp_sum(l) + expf(-m);
    float inv = 1.f / l;
    for (int64_t j = lane; j < n; j += 32) yr[j] = from_f32<T>(expf(to_f32<T>(xr[j]) - m) * inv);
    return;
  }
  const float zs = NORM == HFAN_SPARSEMAX ? 1.f : 0.5f;
  float t = (xmax - 1.f / zs) * zs;  // zmax - 1 in z units
  float tau = kPosInf;
  bool done = !(xmax > kNegInf);
  for (int it = 0; it < 128 && !done; ++it) {
    TauStats st{0.f, 0.f, 0.f, kPosInf};
    for (int64_t j = lane; j < n; j += 32) tau_accumulate(st, to_f32<T>(xr[j]) * zs, t);
    st.cnt = warp_sum(st.cnt);
    st.s1 = warp_sum(st.s1);
    st.s2 = warp_sum(st.s2);
    st.zmin = warp_min(st.zmin);
    done = tau_step(NORM, st, &t, &tau);
  }
  for (int64_t j = lane; j < n; j += 32) yr[j] = from_f32<T>(sparse_prob(NORM, to_f32<T>(xr[j]) * zs, tau));
}

template <typename T, int NORM>
__global__ void __launch_bounds__(256) rownorm_bwd_kernel(int64_t rows, int64_t n, const T* y,
                                                          int64_t ldy, const T* dy, int64_t lddy,
                                                          T* dx, int64_t lddx) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* yr = y + row * ldy;
  const T* dyr = dy + row * lddy;
  T* dxr = dx + row * lddx;
  // w = y (softmax1), 1[y>0] (sparsemax), sqrt(y) (entmax15); dx = w (dy - sum w dy / norm)
  float num = 0.f, den = 0.f;
  for (int64_t j = lane; j < n; j += 32) {
    float yv = to_f32<T>(yr[j]);
    float w = NORM == HFAN_SOFTMAX1 ? yv : (NORM == HFAN_SPARSEMAX ? (yv != 0.f ? 1.f : 0.f) : sqrtf(yv));
    num = fmaf(w, to_f32<T>(dyr[j]), num);
    den += w;
  }
  num = warp_sum(num);
  den = warp_sum(den);
  float c = NORM == HFAN_SOFTMAX1 ? num : (den > 0.f ? num / den : 0.f);
  for (int64_t j = lane; j < n; j += 32) {
    float yv = to_f32<T>(yr[j]);
    float w = NORM == HFAN_SOFTMAX1 ? yv : (NORM == HFAN_SPARSEMAX ? (yv != 0.f ? 1.f : 0.f) : sqrtf(yv));
    dxr[j] = from_f32<T>(w * (to_f32<T>(dyr[j]) - c));
  }
}

template <typename T>
static cudaError_t fwd_t(int norm, int64_t rows, int64_t n, const void* x, int64_t ldx, void* y,
                         int64_t ldy, cudaStream_t s) {
  dim3 grid((unsigned)((rows + 7) / 8));
  const T* xp = static_cast<const T*>(x);
  T* yp = static_cast<T*>(y);
  if (norm == HFAN_SOFTMAX1) rownorm_fwd_kernel<T, HFAN_SOFTMAX1><<<grid, 256, 0, s>>>(rows, n, xp, ldx, yp, ldy);
  else if (norm == HFAN_SPARSEMAX) rownorm_fwd_kernel<T, HFAN_SPARSEMAX><<<grid, 256, 0, s>>>(rows, n, xp, ldx, yp, ldy);
  else rownorm_fwd_kernel<T, HFAN_ENTMAX15><<<grid, 256, 0, s>>>(rows, n, xp, ldx, yp, ldy);
  return cudaGetLastError();
}

template <typename T>
static cudaError_t bwd_t(int norm, int64_t rows, int64_t n, const void* y, int64_t ldy,
                         const void* dy, int64_t lddy, void* dx, int64_t lddx, cudaStream_t s) {
  dim3 grid((unsigned)((rows + 7) / 8));
  const T* yp = static_cast<const T*>(y);
  const T* dyp = static_cast<const T*>(dy);
  T* dxp = static_cast<T*>(dx);
  if (norm == HFAN_SOFTMAX1) rownorm_bwd_kernel<T, HFAN_SOFTMAX1><<<grid, 256, 0, s>>>(rows, n, yp, ldy, dyp, lddy, dxp, lddx);
  else if (norm == HFAN_SPARSEMAX) rownorm_bwd_kernel<T, HFAN_SPARSEMAX><<<grid, 256, 0, s>>>(rows, n, yp, ldy, dyp, lddy, dxp, lddx);
  else rownorm_bwd_kernel<T, HFAN_ENTMAX15><<<grid, 256, 0, s>>>(rows, n, yp, ldy, dyp, lddy, dxp, lddx);
  return cudaGetLastError();
}

cudaError_t rownorm_fwd(int norm, int dtype, int64_t rows, int64_t n, const void* x, int64_t ldx,
                        void* y, int64_t ldy, cudaStream_t s) {
  switch (dtype) {
    case HFAN_FLOAT32: return fwd_t<float>(norm, rows, n, x, ldx, y, ldy, s);
    case HFAN_FLOAT16: return fwd_t<__half>(norm, rows, n, x, ldx, y, ldy, s);
    default: return fwd_t<__nv_bfloat16>(norm, rows, n, x, ldx, y, ldy, s);
  }
}

cudaError_t rownorm_bwd(int norm, int dtype, int64_t rows, int64_t n, const void* y, int64_t ldy,
                        const void* dy, int64_t lddy, void* dx, int64_t lddx, cudaStream_t s) {
  switch (dtype) {
    case HFAN_FLOAT32: return bwd_t<float>(norm, rows, n, y, ldy, dy, lddy, dx, lddx, s);
    case HFAN_FLOAT16: return bwd_t<__half>(norm, rows, n, y, ldy, dy, lddy, dx, lddx, s);
    default: return bwd_t<__nv_bfloat16>(norm, rows, n, y, ldy, dy, lddy, dx, lddx, s);
  }
}

}  // namespace hfan
